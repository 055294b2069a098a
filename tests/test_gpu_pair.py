"""GPU tests of the pair protocol (publish -> wait_armed -> push -> wait_done).

On one GPU, two endpoints (ranks 0 and 1) share the device and every step
runs in order on ONE stream, so each bounded wait is satisfied by a kernel
that finished before it started. On two GPUs the same protocol runs across
NVLink, in one process (peer pointers) and in two processes (CUDA IPC,
handles exchanged over gloo) through the public swap_in API.
"""
import ctypes
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

from lmpool_b200 import _capi
from lmpool_b200.endpoint import TransferEndpoint
from lmpool_b200.layout import affine_layout
from oracle import c_oracle
from tests import kvgen
from tests.conftest import device_count

pytestmark = pytest.mark.gpu


def _same_bits(a, b) -> bool:
    a, b = a.detach().contiguous().cpu(), b.detach().contiguous().cpu()
    return a.shape == b.shape and torch.equal(a.view(torch.uint8), b.view(torch.uint8))


def _pair(dev0: int, dev1: int, shape, seed: int):
    N = shape[2]
    src_cpu = kvgen.seeded_cache(shape, seed)
    dst_cpu = kvgen.seeded_cache(shape, seed + 1)
    src = src_cpu.to(torch.device("cuda", dev0))
    dst = dst_cpu.to(torch.device("cuda", dev1))
    ep0 = TransferEndpoint(0, 2, dev0, N)
    ep1 = TransferEndpoint(1, 2, dev1, N)
    ep0.set_cache(affine_layout(src, shape[1]), src)
    ep1.set_cache(affine_layout(dst, shape[1]), dst)
    link01 = ep0.link(ep1.export_record())
    link10 = ep1.link(ep0.export_record())
    return src_cpu, dst_cpu, src, dst, ep0, ep1, link01, link10


def _ids(ids, dev):
    return torch.tensor(ids, dtype=torch.int64, device=torch.device("cuda", dev))


@pytest.mark.parametrize("variant", [1, 2], ids=["register", "bulk"])
def test_loopback_protocol_on_one_stream(require_gpu, variant):
    lib = require_gpu
    old = _capi.Tuning()
    lib.kvx_get_tuning(ctypes.byref(old))
    lib.kvx_set_tuning(ctypes.byref(_capi.Tuning(variant=variant)))
    try:
        shape = (2, 36, 24, 256, 8, 128)   # Qwen3-8B geometry, reduced N
        src_cpu, dst_cpu, src, dst, ep0, ep1, link01, link10 = _pair(0, 0, shape, 5)
        s = torch.cuda.current_stream(0)
        for round_ in range(3):             # tokens 1, 2, 3 on the same pair
            src_ids = kvgen.seeded_perm(24, 50 + round_)[:8]
            dst_ids = kvgen.seeded_perm(24, 60 + round_)[:8]
            ep0.status.zero_()
            ep1.status.zero_()
            token = ep1.next_token(0)
            assert token == round_ + 1
            ep1.publish(link10, _ids(dst_ids, 0), 8, token, s)
            ep0.wait_armed(link01, 8, 5.0, s)
            ep0.push(ep0.cache, [(link01, link01.cache, _ids(src_ids, 0), 8)], s)
            ep1.wait_done(0, token, 5.0, s)
            ep0.check_status(s, "source")
            ep1.check_status(s, "destination")
            c_oracle.swap_planned(src_cpu, src_ids, dst_cpu, dst_ids, nthreads=4)
            assert _same_bits(dst, dst_cpu)
            assert _same_bits(src, src_cpu)
            assert ep1.read_done(0) == token
        ep0.close()
        ep1.close()
    finally:
        lib.kvx_set_tuning(ctypes.byref(old))


def test_wait_times_out_with_a_status_and_the_context_survives(require_gpu):
    shape = (2, 2, 8, 16, 1, 64)
    _, _, src, dst, ep0, ep1, link01, link10 = _pair(0, 0, shape, 7)
    s = torch.cuda.current_stream(0)
    ep1.status.zero_()
    t0 = time.perf_counter()
    ep1.wait_done(0, 1, 0.2, s)          # nothing will ever signal token 1
    with pytest.raises(_capi.KvxError, match="timed out"):
        ep1.check_status(s, "destination", peers=(0,))
    assert time.perf_counter() - t0 < 30
    assert link10.poisoned                # the pair refuses further use
    with pytest.raises(RuntimeError, match="disabled"):
        ep1.get_link(0)
    ep0.status.zero_()
    ep0.wait_armed(link01, 4, 0.2, s)    # no arm was ever posted
    with pytest.raises(_capi.KvxError, match="timed out"):
        ep0.check_status(s, "source")
    # the device still works
    x = torch.arange(10, device="cuda:0")
    assert int(x.sum().item()) == 45
    ep0.close()
    ep1.close()


def test_stale_completion_cannot_satisfy_a_newer_transfer(require_gpu):
    shape = (2, 2, 8, 16, 1, 64)
    _, _, src, dst, ep0, ep1, link01, link10 = _pair(0, 0, shape, 8)
    s = torch.cuda.current_stream(0)
    ids = _ids([1, 2], 0)
    for e in (ep0, ep1):
        e.status.zero_()
    t1 = ep1.next_token(0)
    ep1.publish(link10, ids, 2, t1, s)
    ep0.wait_armed(link01, 2, 2.0, s)
    ep0.push(ep0.cache, [(link01, link01.cache, ids, 2)], s)
    ep1.wait_done(0, t1, 2.0, s)
    ep1.check_status(s, "first")
    t2 = ep1.next_token(0)                # destination arms again, source never pushes
    ep1.publish(link10, ids, 2, t2, s)
    ep1.wait_done(0, t2, 0.2, s)
    with pytest.raises(_capi.KvxError, match="timed out"):
        ep1.check_status(s, "second")
    ep0.close()
    ep1.close()


def test_count_mismatch_fails_both_sides_without_moving_data(require_gpu):
    shape = (2, 2, 8, 16, 1, 64)
    _, dst_cpu, src, dst, ep0, ep1, link01, link10 = _pair(0, 0, shape, 9)
    s = torch.cuda.current_stream(0)
    for e in (ep0, ep1):
        e.status.zero_()
    token = ep1.next_token(0)
    ep1.publish(link10, _ids([0, 1, 2], 0), 3, token, s)
    ep0.wait_armed(link01, 4, 2.0, s)                       # source moves 4, destination posted 3
    ep0.push(ep0.cache, [(link01, link01.cache, _ids([4, 5, 6, 7], 0), 4)], s)
    ep1.wait_done(0, token, 2.0, s)
    with pytest.raises(_capi.KvxError, match="different block count"):
        ep0.check_status(s, "source")
    with pytest.raises(_capi.KvxError, match="peer reported failure"):
        ep1.check_status(s, "destination")
    assert _same_bits(dst, dst_cpu)
    ep0.close()
    ep1.close()


@pytest.mark.skipif(device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("variant", [1, 2], ids=["register", "bulk"])
def test_two_gpus_one_process_push_over_nvlink(require_gpu, variant):
    lib = require_gpu
    old = _capi.Tuning()
    lib.kvx_get_tuning(ctypes.byref(old))
    lib.kvx_set_tuning(ctypes.byref(_capi.Tuning(variant=variant)))
    try:
        shape = (2, 36, 64, 256, 8, 128)
        src_cpu, dst_cpu, src, dst, ep0, ep1, link01, link10 = _pair(0, 1, shape, 11)
        s0, s1 = torch.cuda.current_stream(0), torch.cuda.current_stream(1)
        src_ids = list(range(10, 26))                 # a contiguous run
        dst_ids = kvgen.seeded_perm(64, 12)[:16]
        ep0.status.zero_()
        ep1.status.zero_()
        token = ep1.next_token(0)
        ep1.publish(link10, _ids(dst_ids, 1), 16, token, s1)
        ep1.wait_done(0, token, 10.0, s1)
        ep0.wait_armed(link01, 16, 10.0, s0)
        ep0.push(ep0.cache, [(link01, link01.cache, _ids(src_ids, 0), 16)], s0)
        ep0.check_status(s0, "source")
        ep1.check_status(s1, "destination")
        c_oracle.swap_planned(src_cpu, src_ids, dst_cpu, dst_ids, nthreads=8)
        assert _same_bits(dst, dst_cpu)
        ep0.close()
        ep1.close()
    finally:
        lib.kvx_set_tuning(ctypes.byref(old))


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _swap_worker(rank: int, port: int, queue) -> None:
    import torch.distributed as dist

    from lmpool_b200 import kv_transfer as kt

    try:
        torch.cuda.set_device(rank)
        os.environ["LOCAL_RANK"] = str(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", world_size=2, rank=rank)
        shape = (2, 4, 16, 2, 1, 8)
        cache = torch.zeros(shape, dtype=torch.float32, device=f"cuda:{rank}")
        kt.register_kv_cache(cache, 4)
        obs = kt.prewarm_p2p_pairs([(0, 1)], num_layers=4, block_size=2, num_kv_heads=1, head_dim=8, num_blocks=2,
                                   dtype=torch.float32, timeout_s=20)
        # reference test (tests/test_kv_transfer.py:105-174): rank 0 blocks [0, 1] -> rank 1 blocks [2, 3]
        if rank == 0:
            cache[0, :, 0].fill_(1.0)
            cache[1, :, 0].fill_(1.5)
            cache[0, :, 1].fill_(2.0)
            cache[1, :, 1].fill_(2.5)
        dist.barrier()
        got = kt.swap_in(remote_gpu=0, remote_blocks=[0, 1], local_gpu=1, kv_cache=cache, num_layers=4,
                         block_size=2, num_kv_heads=1, head_dim=8,
                         local_target_blocks=[2, 3] if rank == 1 else None, negotiate_blocks=False, timeout_s=20)
        dist.barrier()
        ok = got == ([0, 1] if rank == 0 else [2, 3])
        if rank == 1:
            ok &= bool((cache[0, :, 2] == 1.0).all() and (cache[1, :, 2] == 1.5).all())
            ok &= bool((cache[0, :, 3] == 2.0).all() and (cache[1, :, 3] == 2.5).all())
            ok &= bool(cache[:, :, [0, 1] + list(range(4, 16))].abs().sum().item() == 0)
        # seeded bf16 transfers at Qwen3-8B geometry (reduced N), both directions
        # in turn; every rank keeps a CPU model of both caches (the second
        # transfer may read blocks the first one wrote)
        big_shape = (2, 36, 32, 256, 8, 128)
        model = [kvgen.seeded_cache(big_shape, r) for r in range(2)]
        big = model[rank].to(f"cuda:{rank}")
        kt.shutdown()
        kt.register_kv_cache(big, 36)
        kt.prewarm_p2p_pairs([(0, 1)], num_layers=36, block_size=256, num_kv_heads=8, head_dim=128,
                             num_blocks=2, dtype=torch.bfloat16, timeout_s=20)
        for step, (s_rank, d_rank) in enumerate(((0, 1), (1, 0), (0, 1))):
            src_ids = kvgen.seeded_perm(32, 100 + step)[:9]
            dst_ids = kvgen.seeded_perm(32, 200 + step)[:9]
            kt.swap_in(remote_gpu=s_rank, remote_blocks=src_ids, local_gpu=d_rank, kv_cache=big, num_layers=36,
                       block_size=256, num_kv_heads=8, head_dim=128,
                       local_target_blocks=dst_ids if rank == d_rank else None, negotiate_blocks=False,
                       timeout_s=20)
            dist.barrier()
            c_oracle.swap_planned(model[s_rank], src_ids, model[d_rank], dst_ids, nthreads=8)
            ok &= _same_bits(big, model[rank])
        kt.shutdown()
        dist.barrier()
        queue.put({"rank": rank, "ok": bool(ok), "obs": obs})
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001 - report to the parent
        queue.put({"rank": rank, "ok": False, "error": repr(exc)})
        raise


@pytest.mark.skipif(device_count() < 2, reason="needs 2 GPUs")
def test_two_processes_public_api_swap_in(require_gpu):
    ctx = mp.get_context("spawn")
    port = _free_port()
    queue = ctx.Queue()
    procs = [ctx.Process(target=_swap_worker, args=(r, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = []
    deadline = time.time() + 300
    try:
        while len(results) < 2 and time.time() < deadline:
            try:
                results.append(queue.get(timeout=1))
            except Exception:  # noqa: BLE001 - queue.Empty
                if any(p.exitcode not in (None, 0) for p in procs):
                    break
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
                p.join(timeout=10)
    assert len(results) == 2, results
    assert all(r["ok"] for r in results), results
    obs = next(r["obs"] for r in results if r["rank"] == 0)
    assert len(obs) == 1 and obs[0]["src_gpu"] == 0 and obs[0]["dst_gpu"] == 1
    assert obs[0]["transfer_bytes"] == 4 * 2 * 2 * 2 * 1 * 8 * 4


@pytest.mark.parametrize("variant", [1, 2], ids=["register", "bulk"])
def test_one_push_launch_serves_several_destinations(require_gpu, variant):
    """Rank 0 pushes to ranks 1, 2 and 3 in ONE launch (one CTA group and one
    completion counter per destination); all four endpoints share the GPU and
    every step runs in order on one stream."""
    lib = require_gpu
    old = _capi.Tuning()
    lib.kvx_get_tuning(ctypes.byref(old))
    lib.kvx_set_tuning(ctypes.byref(_capi.Tuning(variant=variant)))
    try:
        shape = (2, 6, 20, 64, 4, 64)
        N = shape[2]
        cpus = [kvgen.seeded_cache(shape, 400 + r) for r in range(4)]
        gpus = [c.to("cuda:0") for c in cpus]
        eps = [TransferEndpoint(r, 4, 0, N) for r in range(4)]
        for r in range(4):
            eps[r].set_cache(affine_layout(gpus[r], shape[1]), gpus[r])
        recs = [e.export_record() for e in eps]
        out_links = {d: eps[0].link(recs[d]) for d in (1, 2, 3)}
        in_links = {d: eps[d].link(recs[0]) for d in (1, 2, 3)}
        s = torch.cuda.current_stream(0)
        counts = {1: 5, 2: 0, 3: 9}                      # an empty transfer still completes
        src_ids = {d: kvgen.seeded_perm(N, 410 + d)[:counts[d]] for d in (1, 2, 3)}
        dst_ids = {d: kvgen.seeded_perm(N, 420 + d)[:counts[d]] for d in (1, 2, 3)}
        for e in eps:
            e.status.zero_()
        tokens = {}
        for d in (1, 2, 3):
            tokens[d] = eps[d].next_token(0)
            eps[d].publish(in_links[d], _ids(dst_ids[d], 0), counts[d], tokens[d], s)
        for d in (1, 2, 3):
            eps[0].wait_armed(out_links[d], counts[d], 5.0, s)
        eps[0].push(eps[0].cache, [(out_links[d], out_links[d].cache, _ids(src_ids[d], 0), counts[d])
                                   for d in (1, 2, 3)], s)
        for d in (1, 2, 3):
            eps[d].wait_done(0, tokens[d], 5.0, s)
        for e in eps:
            e.check_status(s, f"rank {e.rank}")
        for d in (1, 2, 3):
            c_oracle.swap_planned(cpus[0], src_ids[d], cpus[d], dst_ids[d], nthreads=4)
            assert _same_bits(gpus[d], cpus[d]), f"destination {d}"
        assert _same_bits(gpus[0], cpus[0])
        for e in eps:
            e.close_links()
        for e in eps:
            e.close()
    finally:
        lib.kvx_set_tuning(ctypes.byref(old))


class _FakeLayer(torch.nn.Module):
    pass


def _fake_runner(rank: int, cache: torch.Tensor):
    from lmpool_b200.model_runner import B200KVTransferMixin

    class Runner(B200KVTransferMixin):
        pass

    r = Runner()
    r.rank = rank
    r.block_size = cache.shape[3]
    r.config = {"num_layers": cache.shape[1], "num_kv_heads": cache.shape[4], "head_dim": cache.shape[5]}
    r.model = torch.nn.ModuleList([_FakeLayer() for _ in range(cache.shape[1])])
    for layer, module in enumerate(r.model):
        module.k_cache = cache[0, layer]
        module.v_cache = cache[1, layer]
    return r


def _api_worker(rank: int, port: int, queue, mode: str = "pull") -> None:
    """Rest of the drop-in surface across two processes: ModelRunner mixin,
    negotiated swap_in, legacy swap_out, swap_batch both ways at once (in the
    process's mode, then with mode="auto": a push round both ways, a pull
    round one way)."""
    os.environ["LMPOOL_B200_KV_MODE"] = mode
    import torch.distributed as dist

    from lmpool_b200 import kv_transfer as kt

    try:
        torch.cuda.set_device(rank)
        os.environ["LOCAL_RANK"] = str(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", world_size=2, rank=rank)
        shape = (2, 8, 40, 64, 8, 128)
        model = [kvgen.seeded_cache(shape, 500 + r) for r in range(2)]
        cache = model[rank].to(f"cuda:{rank}")
        runner = _fake_runner(rank, cache)
        runner.register_kv_cache_for_transfer()
        kt.prewarm_p2p_pairs([(0, 1)], num_layers=8, block_size=64, num_kv_heads=8, head_dim=128, num_blocks=2,
                             dtype=torch.bfloat16, timeout_s=20)
        errors = []
        chunk = 64 * 8 * 128 * 2
        if runner.kv_transfer_bytes(3) != 3 * 8 * 2 * chunk:
            errors.append("kv_transfer_bytes")

        def check(step):
            dist.barrier()
            if not _same_bits(cache, model[rank]):
                errors.append(f"cache differs after {step}")

        # 1. ModelRunner boundary (model_runner.py:747-806)
        src, dst = kvgen.seeded_perm(40, 510)[:6], kvgen.seeded_perm(40, 511)[:6]
        if rank == 0:
            got = runner.execute_swap_out(src, 1)
            if got != src:
                errors.append(f"execute_swap_out returned {got}")
        else:
            got = runner.execute_swap_in(0, src, local_target_blocks=dst)
            if got != dst:
                errors.append(f"execute_swap_in returned {got}")
        c_oracle.swap_planned(model[0], src, model[1], dst, nthreads=4)
        check("execute_swap_out/in")
        # 2. negotiated swap_in (kv_transfer.py:438-452): destination specifies targets
        src, dst = kvgen.seeded_perm(40, 520)[:4], kvgen.seeded_perm(40, 521)[:4]
        got = kt.swap_in(remote_gpu=1, remote_blocks=src, local_gpu=0, kv_cache=cache, num_layers=8,
                         block_size=64, num_kv_heads=8, head_dim=128,
                         local_target_blocks=dst if rank == 0 else None, negotiate_blocks=True, timeout_s=20)
        if got != dst:
            errors.append(f"negotiated swap_in returned {got} on rank {rank}")
        c_oracle.swap_planned(model[1], src, model[0], dst, nthreads=4)
        check("negotiated swap_in")
        # 3. legacy swap_out (kv_transfer.py:310-392): the source names the targets
        src, dst = kvgen.seeded_perm(40, 530)[:5], kvgen.seeded_perm(40, 531)[:5]
        got = kt.swap_out(local_gpu=0, blocks_to_evict=src, target_gpu=1, kv_cache=cache, num_layers=8,
                          block_size=64, num_kv_heads=8, head_dim=128,
                          target_free_blocks=dst if rank == 0 else None, timeout_s=20)
        if got != dst:
            errors.append(f"swap_out returned {got} on rank {rank}")
        c_oracle.swap_planned(model[0], src, model[1], dst, nthreads=4)
        check("swap_out")
        # 4. both directions at once
        perm = kvgen.seeded_perm(40, 540)
        out0, out1 = perm[:7], perm[7:14]          # sources on ranks 0 and 1
        in1, in0 = perm[20:27], perm[27:34]         # targets on ranks 1 and 0 (disjoint from the sources)
        if rank == 0:
            kt.swap_batch([(1, out0)], [(1, out1, in0)], timeout_s=20)
        else:
            kt.swap_batch([(0, out1)], [(0, out0, in1)], timeout_s=20)
        new0, new1 = model[0].clone(), model[1].clone()
        c_oracle.swap_planned(model[0], out0, new1, in1, nthreads=4)
        c_oracle.swap_planned(model[1], out1, new0, in0, nthreads=4)
        model[0], model[1] = new0, new1
        check("swap_batch")
        # 5. mode="auto": both ways at once (a push round), then one way (a pull round)
        perm = kvgen.seeded_perm(40, 550)
        out0, out1, in1, in0 = perm[:5], perm[5:10], perm[20:25], perm[25:30]
        if rank == 0:
            kt.swap_batch([(1, out0)], [(1, out1, in0)], timeout_s=20, mode="auto")
        else:
            kt.swap_batch([(0, out1)], [(0, out0, in1)], timeout_s=20, mode="auto")
        new0, new1 = model[0].clone(), model[1].clone()
        c_oracle.swap_planned(model[0], out0, new1, in1, nthreads=4)
        c_oracle.swap_planned(model[1], out1, new0, in0, nthreads=4)
        model[0], model[1] = new0, new1
        check("swap_batch auto, both ways")
        src, dst = perm[30:34], perm[34:38]
        if rank == 0:
            kt.swap_batch([(1, src)], [], timeout_s=20, mode="auto")
        else:
            kt.swap_batch([], [(0, src, dst)], timeout_s=20, mode="auto")
        c_oracle.swap_planned(model[0], src, model[1], dst, nthreads=4)
        check("swap_batch auto, one way")
        kt.shutdown()
        queue.put({"rank": rank, "errors": errors})
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001
        queue.put({"rank": rank, "errors": [repr(exc)]})
        raise


@pytest.mark.skipif(device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["pull", "push"])
def test_two_processes_drop_in_api_surface(require_gpu, mode):
    ctx = mp.get_context("spawn")
    port = _free_port()
    queue = ctx.Queue()
    procs = [ctx.Process(target=_api_worker, args=(r, port, queue, mode)) for r in range(2)]
    for p in procs:
        p.start()
    results = []
    deadline = time.time() + 300
    try:
        while len(results) < 2 and time.time() < deadline:
            try:
                results.append(queue.get(timeout=1))
            except Exception:  # noqa: BLE001 - queue.Empty
                if any(p.exitcode not in (None, 0) for p in procs):
                    break
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
                p.join(timeout=10)
    assert len(results) == 2, results
    assert all(not r["errors"] for r in results), results


def _all_partner_worker(rank: int, world: int, port: int, queue, mode: str, schedule: str) -> None:
    """Every rank gives blocks to every other rank in one swap_batch call;
    each rank checks its whole cache against the oracle's model of all ranks."""
    import torch.distributed as dist

    from lmpool_b200 import kv_transfer as kt

    try:
        torch.cuda.set_device(rank)
        os.environ["LOCAL_RANK"] = str(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", world_size=world, rank=rank)
        N, B = 48, 3
        shape = (2, 4, N, 16, 2, 64)
        model = [kvgen.seeded_cache(shape, 600 + r) for r in range(world)]
        cache = model[rank].to(f"cuda:{rank}")
        kt.register_kv_cache(cache, 4)
        pairs = [(a, b) for a in range(world) for b in range(a + 1, world)]
        kt.prewarm_p2p_pairs(pairs, num_layers=4, block_size=16, num_kv_heads=2, head_dim=64, num_blocks=2,
                             dtype=torch.bfloat16, timeout_s=20)
        errors = []
        for call in range(2):
            # per rank: targets for each source first, then a pool the sources come from
            perms = [kvgen.seeded_perm(N, 610 + 10 * call + r) for r in range(world)]
            targets = {(a, b): perms[b][a * B:(a + 1) * B] for a in range(world) for b in range(world) if a != b}
            sources = {(a, b): perms[a][world * B + b * B:world * B + (b + 1) * B]
                       for a in range(world) for b in range(world) if a != b}
            peers = [x for x in range(world) if x != rank]
            kt.swap_batch([(d, sources[(rank, d)]) for d in peers],
                          [(s_, sources[(s_, rank)], targets[(s_, rank)]) for s_ in peers],
                          timeout_s=20, mode=mode, schedule=schedule)
            new = [m.clone() for m in model]
            for (a, b), src_ids in sources.items():
                c_oracle.swap_planned(model[a], src_ids, new[b], targets[(a, b)], nthreads=2)
            model = new
            dist.barrier()
            if not _same_bits(cache, model[rank]):
                errors.append(f"cache of rank {rank} differs after call {call}")
        kt.shutdown()
        queue.put({"rank": rank, "errors": errors})
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001
        queue.put({"rank": rank, "errors": [repr(exc)]})
        raise


@pytest.mark.skipif(device_count() < 3, reason="needs 3 GPUs")
@pytest.mark.parametrize("schedule", ["rotated", "concurrent"])
@pytest.mark.parametrize("mode", ["pull", "push"])
def test_all_partner_swap_batch_matches_oracle(require_gpu, mode, schedule):
    world = min(device_count(), 4)
    ctx = mp.get_context("spawn")
    port = _free_port()
    queue = ctx.Queue()
    procs = [ctx.Process(target=_all_partner_worker, args=(r, world, port, queue, mode, schedule))
             for r in range(world)]
    for p in procs:
        p.start()
    results = []
    deadline = time.time() + 300
    try:
        while len(results) < world and time.time() < deadline:
            try:
                results.append(queue.get(timeout=1))
            except Exception:  # noqa: BLE001 - queue.Empty
                if any(p.exitcode not in (None, 0) for p in procs):
                    break
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
                p.join(timeout=10)
    assert len(results) == world, results
    assert all(not r["errors"] for r in results), results


# -- destination-driven (pull) mode ------------------------------------------------

def _pull_steps(ep_dst, link_to_src, ep_src, link_to_dst, sids, dids, n, s_dst, s_src, timeout=5.0,
                grant=True, wait_pulled=True):
    """One pull transfer in dependency order: request (destination), grant
    (source), wait for the grant + pull (destination), wait_pulled (source).
    On one stream every wait is satisfied by a kernel that finished before
    it; on two GPUs each wait is satisfied by a launch issued before it."""
    token = ep_dst.next_token(ep_src.rank)
    ep_dst.request(link_to_src, n, token, s_dst)
    if grant:
        ep_src.grant(link_to_dst, n, timeout, s_src)
    ep_dst.wait_done(ep_src.rank, token, timeout if grant else 0.2, s_dst)
    ep_dst.pull(ep_dst.cache, [(link_to_src, link_to_src.cache, sids, dids, n, token)], s_dst)
    if wait_pulled:
        ep_src.wait_pulled(ep_dst.rank, timeout, s_src)
    return token


@pytest.mark.parametrize("variant", [1, 2], ids=["register", "bulk"])
def test_loopback_pull_on_one_stream(require_gpu, variant):
    """Rank 1 pulls rank 0's blocks (same GPU) and signals rank 0, which waits
    afterwards on the same stream; three rounds on one pair."""
    lib = require_gpu
    old = _capi.Tuning()
    lib.kvx_get_tuning(ctypes.byref(old))
    lib.kvx_set_tuning(ctypes.byref(_capi.Tuning(variant=variant)))
    try:
        shape = (2, 36, 24, 256, 8, 128)
        src_cpu, dst_cpu, src, dst, ep0, ep1, link01, link10 = _pair(0, 0, shape, 15)
        s = torch.cuda.current_stream(0)
        for round_ in range(3):
            src_ids = kvgen.seeded_perm(24, 70 + round_)[:8]
            src_ids[3] = src_ids[0]                          # a repeated source id is legal
            dst_ids = kvgen.seeded_perm(24, 80 + round_)[:8]
            ep0.status.zero_()
            ep1.status.zero_()
            _pull_steps(ep1, link10, ep0, link01, _ids(src_ids, 0), _ids(dst_ids, 0), 8, s, s)
            ep1.check_status(s, "destination")
            ep0.check_status(s, "source")
            c_oracle.swap_planned(src_cpu, src_ids, dst_cpu, dst_ids, nthreads=4)
            assert _same_bits(dst, dst_cpu)
            assert _same_bits(src, src_cpu)
        ep0.close()
        ep1.close()
    finally:
        lib.kvx_set_tuning(ctypes.byref(old))


def test_one_pull_launch_reads_several_sources(require_gpu):
    shape = (2, 5, 20, 64, 4, 64)
    N = shape[2]
    cpus = [kvgen.seeded_cache(shape, 600 + r) for r in range(4)]
    gpus = [c.to("cuda:0") for c in cpus]
    eps = [TransferEndpoint(r, 4, 0, N) for r in range(4)]
    for r in range(4):
        eps[r].set_cache(affine_layout(gpus[r], shape[1]), gpus[r])
    recs = [e.export_record() for e in eps]
    to_src = {r: eps[3].link(recs[r]) for r in (0, 1, 2)}
    for r in (0, 1, 2):
        eps[r].link(recs[3])
    s = torch.cuda.current_stream(0)
    counts = {0: 6, 1: 0, 2: 4}
    perm = kvgen.seeded_perm(N, 610)
    dst_ids = {0: perm[0:6], 1: [], 2: perm[6:10]}                # disjoint targets
    src_ids = {r: kvgen.seeded_perm(N, 620 + r)[:counts[r]] for r in (0, 1, 2)}
    for e in eps:
        e.status.zero_()
    tokens = {r: eps[3].next_token(r) for r in (0, 1, 2)}
    for r in (0, 1, 2):
        eps[3].request(to_src[r], counts[r], tokens[r], s)
    for r in (0, 1, 2):
        eps[r].grant(eps[r].get_link(3), counts[r], 5.0, s)
    for r in (0, 1, 2):
        eps[3].wait_done(r, tokens[r], 5.0, s)
    eps[3].pull(eps[3].cache, [(to_src[r], to_src[r].cache, _ids(src_ids[r], 0), _ids(dst_ids[r], 0), counts[r],
                                tokens[r]) for r in (0, 1, 2)], s)
    for r in (0, 1, 2):
        eps[r].wait_pulled(3, 5.0, s)
    for e in eps:
        e.check_status(s, f"rank {e.rank}")
    for r in (0, 1, 2):
        c_oracle.swap_planned(cpus[r], src_ids[r], cpus[3], dst_ids[r], nthreads=4)
    assert _same_bits(gpus[3], cpus[3])
    for r in (0, 1, 2):
        assert _same_bits(gpus[r], cpus[r])
    for e in eps:
        e.close_links()
    for e in eps:
        e.close()


def test_wait_pulled_times_out_and_stale_pulls_do_not_count(require_gpu):
    shape = (2, 2, 8, 16, 1, 64)
    _, _, src, dst, ep0, ep1, link01, link10 = _pair(0, 0, shape, 16)
    s = torch.cuda.current_stream(0)
    ep0.status.zero_()
    ep0.wait_pulled(1, 0.2, s)                  # nothing pulled yet
    with pytest.raises(_capi.KvxError, match="timed out"):
        ep0.check_status(s, "source")
    ep0.status.zero_()
    ep1.status.zero_()
    ids = _ids([1, 2], 0)
    _pull_steps(ep1, link10, ep0, link01, ids, ids, 2, s, s, timeout=2.0)   # consumes that pull
    ep0.check_status(s, "first")
    ep0.wait_pulled(1, 0.2, s)                  # the same pull cannot satisfy a second wait
    with pytest.raises(_capi.KvxError, match="timed out"):
        ep0.check_status(s, "second")
    ep0.close()
    ep1.close()


@pytest.mark.skipif(device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("variant", [1, 2], ids=["register", "bulk"])
def test_two_gpus_one_process_pull_over_nvlink(require_gpu, variant):
    lib = require_gpu
    old = _capi.Tuning()
    lib.kvx_get_tuning(ctypes.byref(old))
    lib.kvx_set_tuning(ctypes.byref(_capi.Tuning(variant=variant)))
    try:
        shape = (2, 36, 64, 256, 8, 128)
        src_cpu, dst_cpu, src, dst, ep0, ep1, link01, link10 = _pair(0, 1, shape, 17)
        s0, s1 = torch.cuda.current_stream(0), torch.cuda.current_stream(1)
        src_ids = kvgen.seeded_perm(64, 18)[:16]
        dst_ids = kvgen.seeded_perm(64, 19)[:16]
        ep0.status.zero_()
        ep1.status.zero_()
        _pull_steps(ep1, link10, ep0, link01, _ids(src_ids, 1), _ids(dst_ids, 1), 16, s1, s0, timeout=10.0)
        ep1.check_status(s1, "destination")
        ep0.check_status(s0, "source")
        c_oracle.swap_planned(src_cpu, src_ids, dst_cpu, dst_ids, nthreads=8)
        assert _same_bits(dst, dst_cpu)
        ep0.close()
        ep1.close()
    finally:
        lib.kvx_set_tuning(ctypes.byref(old))


def test_pull_without_a_grant_moves_nothing_and_reports_failure(require_gpu):
    """A destination whose request is never granted waits (bounded), its
    pull copies nothing, and the source learns of it as a failed pull."""
    shape = (2, 3, 10, 16, 2, 32)
    _, dst_cpu, src, dst, ep0, ep1, link01, link10 = _pair(0, 0, shape, 21)
    s = torch.cuda.current_stream(0)
    ep0.status.zero_()
    ep1.status.zero_()
    ids = _ids([1, 2, 3], 0)
    _pull_steps(ep1, link10, ep0, link01, ids, ids, 3, s, s, grant=False)
    with pytest.raises(_capi.KvxError, match="timed out"):
        ep1.check_status(s, "destination")
    with pytest.raises(_capi.KvxError, match="reported failure"):
        ep0.check_status(s, "source")
    assert _same_bits(dst, dst_cpu)
    ep0.close()
    ep1.close()


def test_push_arm_and_pull_request_never_satisfy_each_other(require_gpu):
    """Two ends that disagree on the mode fail on both sides without moving data."""
    shape = (2, 3, 10, 16, 2, 32)
    _, dst_cpu, src, dst, ep0, ep1, link01, link10 = _pair(0, 0, shape, 22)
    s = torch.cuda.current_stream(0)
    ids = _ids([4, 5], 0)
    # destination pulls, source pushes
    ep0.status.zero_()
    ep1.status.zero_()
    token = ep1.next_token(0)
    ep1.request(link10, 2, token, s)
    ep0.wait_armed(link01, 2, 2.0, s)
    ep0.push(ep0.cache, [(link01, link01.cache, ids, 2)], s)
    ep1.wait_done(0, token, 2.0, s)
    ep1.pull(ep1.cache, [(link10, link10.cache, ids, ids, 2, token)], s)
    with pytest.raises(_capi.KvxError, match="different block count"):
        ep0.check_status(s, "source")
    with pytest.raises(_capi.KvxError, match="reported failure"):
        ep1.check_status(s, "destination")
    assert _same_bits(dst, dst_cpu)
    # destination pushes (publishes ids), source grants a pull
    ep0.status.zero_()
    ep1.status.zero_()
    token = ep1.next_token(0)
    ep1.publish(link10, ids, 2, token, s)
    ep0.grant(link01, 2, 2.0, s)
    ep1.wait_done(0, token, 2.0, s)
    with pytest.raises(_capi.KvxError, match="different block count"):
        ep0.check_status(s, "source")
    with pytest.raises(_capi.KvxError, match="reported failure"):
        ep1.check_status(s, "destination")
    assert _same_bits(dst, dst_cpu)
    ep0.close()
    ep1.close()


def test_a_reset_pair_recovers_after_an_injected_failure(require_gpu):
    """A timeout reported on the host disables the pair; resetting both ends
    (what prewarm does) brings it back from token 1, with no new mailbox."""
    shape = (2, 3, 12, 16, 2, 32)
    src_cpu, dst_cpu, src, dst, ep0, ep1, link01, link10 = _pair(0, 0, shape, 23)
    s = torch.cuda.current_stream(0)
    ids_a = kvgen.seeded_perm(12, 24)[:4]
    for _ in range(3):
        ep0.status.zero_()
        ep1.status.zero_()
        _pull_steps(ep1, link10, ep0, link01, _ids(ids_a, 0), _ids(ids_a, 0), 4, s, s)
        ep1.check_status(s, "destination")
        ep0.check_status(s, "source")
    # inject: the destination's status word reports a bulk-pipeline timeout
    ep1.status.fill_(_capi.DEV_PIPE_TIMEOUT)
    with pytest.raises(_capi.KvxError):
        ep1.check_status(s, "destination", peers=[0])
    with pytest.raises(RuntimeError, match="disabled"):
        ep1.get_link(0)
    for ep, peer in ((ep0, 1), (ep1, 0)):
        ep.reset_pair(peer, s)
    ep0.status.zero_()
    ep1.status.zero_()
    ids_b = kvgen.seeded_perm(12, 25)[:5]
    dst_b = kvgen.seeded_perm(12, 26)[:5]
    token = _pull_steps(ep1, ep1.get_link(0), ep0, ep0.get_link(1), _ids(ids_b, 0), _ids(dst_b, 0), 5, s, s)
    assert token == 1
    ep1.check_status(s, "destination")
    ep0.check_status(s, "source")
    c_oracle.swap_planned(src_cpu, ids_a, dst_cpu, ids_a, nthreads=2)
    c_oracle.swap_planned(src_cpu, ids_b, dst_cpu, dst_b, nthreads=2)
    assert _same_bits(dst, dst_cpu)
    ep0.close()
    ep1.close()


@pytest.mark.skipif(device_count() < 2, reason="needs 2 GPUs")
def test_pull_reads_what_the_source_wrote_before_its_grant(require_gpu):
    """Ordering: the source's stream writes its blocks (a long local move)
    and only then grants; the destination, on another GPU, requests and pulls
    at once. The pulled blocks are the newly written ones, bit for bit."""
    shape = (2, 36, 96, 64, 8, 128)
    src_cpu, dst_cpu, src, dst, ep0, ep1, link01, link10 = _pair(0, 1, shape, 27)
    s0, s1 = torch.cuda.current_stream(0), torch.cuda.current_stream(1)
    staging = kvgen.seeded_perm(96, 28)[:32]
    blocks = kvgen.seeded_perm(96, 29)
    blocks = [b for b in blocks if b not in set(staging)][:32]
    targets = kvgen.seeded_perm(96, 30)[:32]
    status = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    from lmpool_b200 import kv_transfer as kt
    ep0.status.zero_()
    ep1.status.zero_()
    token = ep1.next_token(0)
    ep1.request(link10, 32, token, s1)
    kt._launch_move(0, ep0.cache, ep0.cache, _ids(staging, 0), _ids(blocks, 0), 32, status, s0)
    ep0.grant(link01, 32, 10.0, s0)
    ep1.wait_done(0, token, 10.0, s1)
    ep1.pull(ep1.cache, [(link10, link10.cache, _ids(blocks, 1), _ids(targets, 1), 32, token)], s1)
    ep0.wait_pulled(1, 10.0, s0)
    ep1.check_status(s1, "destination")
    ep0.check_status(s0, "source")
    assert int(status.item()) == 0
    moved = src_cpu.clone()
    moved[:, :, blocks] = src_cpu[:, :, staging]
    c_oracle.swap_planned(moved, blocks, dst_cpu, targets, nthreads=8)
    assert _same_bits(dst, dst_cpu)
    assert _same_bits(src, moved)
    ep0.close()
    ep1.close()


def test_a_deferred_grant_is_read_later_and_a_failed_one_disables_the_pair(require_gpu):
    """The source can return once its grant is enqueued: the grant's outcome
    is read from pinned memory after its event completes. A grant nobody
    requested runs out (bounded) and disables the pair without raising in
    an unrelated call."""
    shape = (2, 3, 12, 16, 2, 32)
    src_cpu, dst_cpu, src, dst, ep0, ep1, link01, link10 = _pair(0, 0, shape, 31)
    s = torch.cuda.current_stream(0)
    ids, targets = kvgen.seeded_perm(12, 32)[:4], kvgen.seeded_perm(12, 33)[:4]
    ep1.status.zero_()
    token = ep1.next_token(0)
    ep1.request(link10, 4, token, s)
    ep0.grant_deferred(link01, 4, 5.0, s, "deferred grant")
    ep1.wait_done(0, token, 5.0, s)
    ep1.pull(ep1.cache, [(link10, link10.cache, _ids(ids, 0), _ids(targets, 0), 4, token)], s)
    ep1.check_status(s, "destination")
    ep0.poll_deferred(wait=True)
    assert link01.poisoned is None and len(ep0._async_free) == ep0.ASYNC_SLOTS
    c_oracle.swap_planned(src_cpu, ids, dst_cpu, targets, nthreads=2)
    assert _same_bits(dst, dst_cpu)
    # a grant with no request: its bounded wait runs out on the device
    ep0.grant_deferred(link01, 4, 0.2, s, "unrequested grant")
    ep0.poll_deferred(wait=True)
    assert link01.poisoned and "timed out" in link01.poisoned
    with pytest.raises(RuntimeError, match="disabled"):
        ep0.get_link(1)
    ep0.close()
    ep1.close()


def test_a_report_left_by_an_earlier_transfer_does_not_satisfy_a_newer_wait(require_gpu):
    """A source that returned once granted leaves its transfer's pull report
    unconsumed. A later transfer's wait for the destination's read must wait
    for that transfer's own report, not take the old one."""
    shape = (2, 3, 12, 16, 2, 32)
    src_cpu, dst_cpu, src, dst, ep0, ep1, link01, link10 = _pair(0, 0, shape, 34)
    s = torch.cuda.current_stream(0)
    ids = kvgen.seeded_perm(12, 35)[:3]
    ep0.status.zero_()
    ep1.status.zero_()
    _pull_steps(ep1, link10, ep0, link01, _ids(ids, 0), _ids(ids, 0), 3, s, s, wait_pulled=False)   # report left behind
    token = ep1.next_token(0)
    ep1.request(link10, 3, token, s)
    ep0.grant(link01, 3, 5.0, s)
    ep0.wait_pulled(1, 0.2, s)                       # the new transfer has not been read yet
    with pytest.raises(_capi.KvxError, match="timed out"):
        ep0.check_status(s, "source")
    ep0.status.zero_()
    ep1.wait_done(0, token, 5.0, s)
    ep1.pull(ep1.cache, [(link10, link10.cache, _ids(ids, 0), _ids(ids, 0), 3, token)], s)
    ep0.wait_pulled(1, 5.0, s)                       # now its own report is there
    ep0.check_status(s, "source")
    ep1.check_status(s, "destination")
    c_oracle.swap_planned(src_cpu, ids, dst_cpu, ids, nthreads=2)
    assert _same_bits(dst, dst_cpu)
    ep0.close()
    ep1.close()
