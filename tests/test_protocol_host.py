"""Host-side orchestration of the pair protocol (TransferEndpoint.exchange),
checked on CPU with the device steps replaced by recorders.

The order of the enqueued steps is what makes every exchange deadlock-free:
in push mode each rank publishes all its arms before it waits for any peer's
arm, and in pull mode each rank issues its pull before it waits for any
peer's report. Tokens come from the destination and grow per source.
"""
import threading

import pytest

from lmpool_b200.endpoint import PeerLink, TransferEndpoint


def _endpoint(rank: int, world: int):
    ep = object.__new__(TransferEndpoint)
    ep.rank, ep.world_size, ep.device = rank, world, 0
    ep.tokens_issued = {}
    ep._lock = threading.Lock()
    ep.links = {r: PeerLink(peer=r, mailbox=None, cache=f"cache{r}") for r in range(world) if r != rank}
    calls = []
    ep.publish = lambda link, ids, n, token, stream: calls.append(("publish", link.peer, n, token))
    ep.wait_armed = lambda link, n, t, stream: calls.append(("wait_armed", link.peer, n))
    ep.push = lambda local, targets, stream: calls.append(
        ("push", [(link.peer, layout, n) for link, layout, _ids, n in targets]))
    ep.wait_done = lambda src, token, t, stream: calls.append(("wait_done", src, token))
    ep.pull = lambda local, sources, stream: calls.append(
        ("pull", [(link.peer, layout, n, token) for link, layout, _s, _d, n, token in sources]))
    ep.wait_pulled = lambda dst, t, stream: calls.append(("wait_pulled", dst))
    ep.request = lambda link, n, token, stream: calls.append(("request", link.peer, n, token))
    ep.grant = lambda link, n, t, stream, status_ptr=None: calls.append(("grant", link.peer, n))
    return ep, calls


def test_push_arms_everything_before_any_wait():
    ep, calls = _endpoint(0, 4)
    ep.exchange("push", "local", [(1, "i1", 5), (2, "i2", 0)], [(1, "s1", "d1", 3), (3, "s3", "d3", 4)], 1.0, None)
    kinds = [c[0] for c in calls]
    assert kinds == ["publish", "publish", "wait_armed", "wait_armed", "push", "wait_done", "wait_done"]
    assert calls[0] == ("publish", 1, 3, 1) and calls[1] == ("publish", 3, 4, 1)
    assert calls[4] == ("push", [(1, "cache1", 5), (2, "cache2", 0)])
    assert calls[5] == ("wait_done", 1, 1) and calls[6] == ("wait_done", 3, 1)


def test_pull_requests_and_grants_everything_before_any_wait():
    ep, calls = _endpoint(2, 4)
    ep.exchange("pull", "local", [(0, "i0", 5)], [(1, "s1", "d1", 3), (3, "s3", "d3", 0)], 1.0, None,
                peer_layouts={3: "payload3"})
    assert [c[0] for c in calls] == ["request", "request", "grant", "wait_done", "wait_done", "pull",
                                     "wait_pulled"]
    assert calls[0] == ("request", 1, 3, 1) and calls[1] == ("request", 3, 0, 1)
    assert calls[2] == ("grant", 0, 5)
    assert calls[3] == ("wait_done", 1, 1) and calls[4] == ("wait_done", 3, 1)
    assert calls[5] == ("pull", [(1, "cache1", 3, 1), (3, "payload3", 0, 1)])
    assert calls[6] == ("wait_pulled", 0)


def test_a_source_that_returns_once_granted_skips_the_read_wait():
    ep, calls = _endpoint(1, 2)
    ep.exchange("pull", "local", [(0, "i0", 2)], [], 1.0, None, wait_pulled=False)
    assert calls == [("grant", 0, 2)]


def test_tokens_grow_per_source_across_exchanges():
    ep, calls = _endpoint(1, 3)
    for _ in range(3):
        ep.exchange("pull", "local", [], [(0, "s", "d", 1)], 1.0, None)
    ep.exchange("push", "local", [], [(0, "s", "d", 1), (2, "s", "d", 1)], 1.0, None)
    tokens_from_0 = [c[1][0][3] for c in calls if c[0] == "pull"] + [c[3] for c in calls if c[:2] == ("publish", 0)]
    assert tokens_from_0 == [1, 2, 3, 4]
    assert [c[3] for c in calls if c[:2] == ("publish", 2)] == [1]


def test_unknown_mode_and_unlinked_peer_are_refused():
    ep, _ = _endpoint(0, 2)
    with pytest.raises(RuntimeError, match="mode"):
        ep.exchange("sideways", "local", [], [], 1.0, None)
    with pytest.raises(RuntimeError, match="no mapping of rank 5"):
        ep.exchange("pull", "local", [(5, "i", 1)], [], 1.0, None)
    ep.links[1].poisoned = "earlier timeout"
    with pytest.raises(RuntimeError, match="disabled"):
        ep.exchange("push", "local", [(1, "i", 1)], [], 1.0, None)


def test_registered_cache_check_accepts_views_and_the_tensor_and_refuses_others():
    import torch

    from lmpool_b200 import kv_transfer as kt
    from lmpool_b200.layout import affine_layout

    t = torch.empty(2, 4, 6, 8, 2, 16, dtype=torch.bfloat16)
    ep = object.__new__(TransferEndpoint)
    ep.cache = affine_layout(t, 4)
    kt._check_registered(ep, t, 4)
    kt._check_registered(ep, [(t[0, layer], t[1, layer]) for layer in range(4)], 4)
    other = torch.empty_like(t)
    with pytest.raises(RuntimeError, match="not the cache registered"):
        kt._check_registered(ep, other, 4)
    with pytest.raises(RuntimeError, match="num_layers"):
        kt._check_registered(ep, t, 3)
    ep.cache = None
    with pytest.raises(RuntimeError, match="no KV cache registered"):
        kt._check_registered(ep, t, 4)


def test_rotated_schedule_runs_one_tournament_round_per_partner():
    """Rounds are a round-robin tournament: both directions of a pair share
    a round, each round gives every rank one partner."""
    from lmpool_b200.endpoint import pair_round

    for n in range(2, 10):
        rounds: dict = {}
        for a in range(n):
            for b in range(a + 1, n):
                r = pair_round(a, b, n)
                assert r == pair_round(b, a, n)
                rounds.setdefault(r, []).append((a, b))
        assert sorted(rounds) == list(range(n - 1 + n % 2))
        for pairs in rounds.values():
            members = [x for pair in pairs for x in pair]
            assert len(members) == len(set(members))
    with pytest.raises(RuntimeError, match="no round"):
        pair_round(1, 1, 4)
    ep, calls = _endpoint(1, 4)
    ep.exchange_rotated("push", "local", [(2, "i2", 5), (0, "i0", 6)], [(3, "s3", "d3", 7), (0, "s0", "d0", 8)],
                        1.0, None)
    # 4 ranks: {1,3} meet in schedule step 1, {1,2} in step 0, {0,1} in step 2: the pair with
    # rank 0 sends and receives in the same round
    kinds = [c[0] for c in calls]
    assert kinds == ["wait_armed", "push",                             # step 0: to 2
                     "publish", "wait_done",                           # step 1: from 3
                     "publish", "wait_armed", "push", "wait_done"]     # step 2: both ways with 0
    assert [c[1] for c in calls if c[0] == "push"] == [[(2, "cache2", 5)], [(0, "cache0", 6)]]
    assert [(c[1], c[2]) for c in calls if c[0] == "publish"] == [(3, 7), (0, 8)]
    with pytest.raises(RuntimeError, match="mode"):
        ep.exchange_rotated("sideways", "local", [], [], 1.0, None)


def test_disjoint_pairs_exchange_both_ways_in_a_single_round():
    """Phase A through the rotated schedule at 4 and 8 ranks: every pair
    sends both ways in one round (one exchange call per rank)."""
    for world in (4, 8):
        for r in range(world):
            ep, calls = _endpoint(r, world)
            partner = r + 1 if r % 2 == 0 else r - 1
            ep.exchange_rotated("push", "local", [(partner, "i", 3)], [(partner, "s", "d", 3)], 1.0, None)
            assert [c[0] for c in calls] == ["publish", "wait_armed", "push", "wait_done"]


def _simulate(streams: dict[int, list], mode: str) -> None:
    """Run every rank's recorded device steps against one another, in any
    interleaving, with the mailbox semantics of the kernels: an arm slot per
    (source, destination) that must be free when published or requested, a
    done token (push completion or pull grant) the destination waits for, a
    pulled report the source waits for. Raises on a deadlock (no rank can
    make progress) or a clobbered mailbox."""
    arm, done, pulled = {}, {}, {}
    pos = {r: 0 for r in streams}
    while any(pos[r] < len(streams[r]) for r in streams):
        progressed = False
        for r, steps in streams.items():
            while pos[r] < len(steps):
                step = steps[pos[r]]
                kind = step[0]
                if kind in ("publish", "request"):    # r is the destination, step[1] the source
                    assert (step[1], r) not in arm, "arm published twice before the source used it"
                    arm[(step[1], r)] = step[3]
                elif kind == "wait_armed":
                    if (r, step[1]) not in arm:
                        break
                elif kind == "grant":                 # r is the source, step[1] the destination
                    if (r, step[1]) not in arm:
                        break
                    done[(r, step[1])] = arm.pop((r, step[1]))
                elif kind == "push":
                    for peer, _layout, _n in step[1]:
                        done[(r, peer)] = arm.pop((r, peer))
                elif kind == "wait_done":
                    if done.get((step[1], r)) != step[2]:
                        break
                    del done[(step[1], r)]
                elif kind == "pull":
                    for peer, _layout, _n, _token in step[1]:
                        pulled[(peer, r)] = pulled.get((peer, r), 0) + 1
                elif kind == "wait_pulled":
                    if not pulled.get((r, step[1])):
                        break
                    pulled[(r, step[1])] -= 1
                pos[r] += 1
                progressed = True
        if not progressed:
            raise AssertionError(f"deadlock ({mode}): " + ", ".join(
                f"rank {r} stuck at {streams[r][pos[r]]}" for r in streams if pos[r] < len(streams[r])))
    assert not arm and not done and not any(pulled.values())


@pytest.mark.parametrize("mode,schedule", [("push", "concurrent"), ("pull", "concurrent"), ("push", "rotated"),
                                           ("pull", "rotated"), ("auto", "rotated")])
@pytest.mark.parametrize("world,seed", [(2, 0), (4, 1), (5, 5), (6, 2), (8, 3), (8, 4)])
def test_every_rank_finishes_for_random_transfer_sets(mode, schedule, world, seed):
    """Any set of directed transfers, each rank calling the same schedule
    several times in a row, completes without a deadlock."""
    import random

    rng = random.Random(seed)
    streams = {}
    eps = {r: _endpoint(r, world) for r in range(world)}
    for _call in range(3):
        pairs = {(a, b) for a in range(world) for b in range(world) if a != b and rng.random() < 0.6}
        for r, (ep, _calls) in eps.items():
            outgoing = [(b, f"i{b}", 1 + rng.randrange(4)) for a, b in sorted(pairs) if a == r]
            incoming = [(a, f"s{a}", f"d{a}", 1) for a, b in sorted(pairs) if b == r]
            getattr(ep, "exchange" if schedule == "concurrent" else "exchange_rotated")(
                mode, "local", outgoing, incoming, 1.0, None)
    for r, (_ep, calls) in eps.items():
        streams[r] = calls
    _simulate(streams, mode)


@pytest.mark.parametrize("mode", ["push", "pull"])
def test_simulator_detects_a_deadlock(mode):
    """Two sequential one-way calls in opposite directions: each rank first
    waits for the other's arm (push) or request (pull)."""
    a, ca = _endpoint(0, 2)
    b, cb = _endpoint(1, 2)
    a.exchange(mode, "local", [(1, "i", 1)], [], 1.0, None)
    a.exchange(mode, "local", [], [(1, "s", "d", 1)], 1.0, None)
    b.exchange(mode, "local", [(0, "i", 1)], [], 1.0, None)
    b.exchange(mode, "local", [], [(0, "s", "d", 1)], 1.0, None)
    with pytest.raises(AssertionError, match="deadlock"):
        _simulate({0: ca, 1: cb}, mode)


def test_sequential_calls_in_one_direction_at_a_time_finish_in_pull_mode():
    """What LMPool issues (one plan per pair at a time): 0->1, then 1->0,
    both ranks calling in the same order, with the source returning once its
    grant is enqueued or after the read."""
    for wait in (True, False):
        a, ca = _endpoint(0, 2)
        b, cb = _endpoint(1, 2)
        a.exchange("pull", "local", [(1, "i", 2)], [], 1.0, None, wait_pulled=wait)
        b.exchange("pull", "local", [], [(0, "s", "d", 2)], 1.0, None)
        b.exchange("pull", "local", [(0, "i", 3)], [], 1.0, None, wait_pulled=wait)
        a.exchange("pull", "local", [], [(1, "s", "d", 3)], 1.0, None)
        streams = {0: ca, 1: cb}
        if not wait:   # the reads nobody waits for leave their reports behind
            streams[0] = ca + [("wait_pulled", 1)]
            streams[1] = cb + [("wait_pulled", 0)]
        _simulate(streams, "pull")


def _batch_setup(monkeypatch):
    """swap_batch up to its first device step: a registered CPU-shaped cache
    on a stub endpoint, peers 1-3 linked with caches of the same shape."""
    import torch

    from lmpool_b200 import kv_transfer as kt
    from lmpool_b200.layout import affine_layout

    lay = affine_layout(torch.empty(2, 2, 10, 4, 1, 8, dtype=torch.bfloat16), 2)
    ep, calls = _endpoint(0, 4)
    ep.cache = lay
    for link in ep.links.values():
        link.cache = lay
    monkeypatch.setattr(kt.dist, "get_rank", lambda: 0)
    monkeypatch.setattr(kt, "_local_device", lambda rank: 0)
    monkeypatch.setitem(kt._ENDPOINTS, 0, ep)

    def no_upload(*a, **k):
        raise AssertionError("reached the device upload")

    monkeypatch.setattr(kt, "_upload", no_upload)
    return kt, calls


def test_swap_batch_refuses_bad_batches_before_any_device_step(monkeypatch):
    kt, calls = _batch_setup(monkeypatch)
    S = "stream"   # no CUDA here: stands in for the caller's stream
    with pytest.raises(RuntimeError, match="more than once in outgoing"):
        kt.swap_batch([(1, [0]), (1, [2])], [])
    with pytest.raises(RuntimeError, match="more than once in incoming"):
        kt.swap_batch([], [(2, [0], [1]), (2, [3], [4])])
    with pytest.raises(RuntimeError, match="schedule"):
        kt.swap_batch([(1, [0])], [], schedule="sideways")
    with pytest.raises(RuntimeError, match="targets of all incoming"):
        kt.swap_batch([], [(1, [0, 1], [5, 6]), (3, [2], [6])], stream=S)   # block 6 written by two sources
    with pytest.raises(RuntimeError, match="3 source ids, 2 targets"):
        kt.swap_batch([], [(1, [0, 1, 2], [5, 6])], stream=S)
    with pytest.raises(RuntimeError, match="outside"):
        kt.swap_batch([(2, [10])], [], stream=S)
    assert calls == []
    with pytest.raises(AssertionError, match="device upload"):     # a good batch gets that far
        kt.swap_batch([(1, [0, 1])], [(1, [2], [7]), (3, [2], [8])], stream=S)


def test_every_enqueued_step_marks_the_status_word_unchecked():
    """reset_status skips the zeroing launch only while the last check read
    zero and nothing was enqueued since; every device step clears that."""
    import torch

    from lmpool_b200 import _capi
    from lmpool_b200.layout import affine_layout

    class Lib:
        def __getattr__(self, name):
            return lambda *args: 0

    lay = affine_layout(torch.empty(2, 1, 4, 2, 1, 8, dtype=torch.bfloat16), 1)
    ep = object.__new__(TransferEndpoint)
    ep.lib, ep.device, ep.rank = Lib(), 0, 0
    ep.mailbox = _capi.Mailbox()
    ep.status = torch.zeros(1, dtype=torch.int32)
    link = PeerLink(peer=1, mailbox=_capi.Mailbox(), cache=lay)
    ids = torch.zeros(2, dtype=torch.int64)
    steps = [
        lambda: ep.request(link, 2, 1, None),
        lambda: ep.grant(link, 2, 1.0, None),
        lambda: ep.publish(link, ids, 2, 1, None),
        lambda: ep.wait_done(1, 1, 1.0, None),
        lambda: ep.wait_armed(link, 2, 1.0, None),
        lambda: ep.push(lay, [(link, lay, ids, 2)], None),
        lambda: ep.pull(lay, [(link, lay, ids, ids, 2, 1)], None),
        lambda: ep.wait_pulled(1, 1.0, None),
    ]
    for step in steps:
        ep.status_clean = True
        step()
        assert ep.status_clean is False


def test_source_return_setting_picks_the_source_side_path(monkeypatch):
    """Pull mode: 'read' runs the whole exchange (grant + wait for the read);
    'granted' only enqueues a deferred grant. Push mode ignores the setting."""
    from lmpool_b200 import kv_transfer as kt

    ep, calls = _endpoint(0, 2)
    ep.mode, ep.cache = "pull", "local"
    ep.grant_deferred = lambda link, n, t, stream, what: calls.append(("grant_deferred", link.peer, n))
    ran = []
    monkeypatch.setattr(kt, "_run_exchange", lambda *a, **k: ran.append(a[2]))
    monkeypatch.setattr(kt, "_upload", lambda device, stream, *arrays: [list(x) for x in arrays])
    monkeypatch.setenv("LMPOOL_B200_SOURCE_RETURN", "granted")
    kt._source_side(ep, 1, [3, 4, 5], 1.0, None)
    assert calls == [("grant_deferred", 1, 3)] and ran == []
    monkeypatch.setenv("LMPOOL_B200_SOURCE_RETURN", "read")
    kt._source_side(ep, 1, [3, 4, 5], 1.0, None)
    assert ran == [[(1, None, 3)]]
    kt._source_side(ep, 1, [3, 4], 1.0, None, wait=False)     # an explicit wait overrides the setting
    assert calls[-1] == ("grant_deferred", 1, 2)
    ep.mode = "push"
    monkeypatch.setenv("LMPOOL_B200_SOURCE_RETURN", "granted")
    kt._source_side(ep, 1, [7], 1.0, None)
    assert ran[-1] == [(1, [7], 1)]
    monkeypatch.setenv("LMPOOL_B200_SOURCE_RETURN", "later")
    ep.mode = "pull"
    with pytest.raises(RuntimeError, match="LMPOOL_B200_SOURCE_RETURN"):
        kt._source_side(ep, 1, [7], 1.0, None)


def test_auto_mode_pushes_two_way_rounds_and_pulls_one_way_rounds():
    ep, calls = _endpoint(1, 4)
    # partner 0 both ways (step 2), partner 2 one way out (step 0), partner 3 one way in (step 1)
    ep.exchange_rotated("auto", "local", [(0, "i0", 2), (2, "i2", 3)], [(0, "s0", "d0", 2), (3, "s3", "d3", 4)],
                        1.0, None)
    kinds = [c[0] for c in calls]
    assert kinds == ["grant", "wait_pulled",                                  # step 0: pull, to 2
                     "request", "wait_done", "pull",                          # step 1: pull, from 3
                     "publish", "wait_armed", "push", "wait_done"]           # step 2: push, both ways with 0


def test_swap_batch_refuses_auto_without_rounds(monkeypatch):
    kt, calls = _batch_setup(monkeypatch)
    with pytest.raises(RuntimeError, match="needs schedule='rotated'"):
        kt.swap_batch([(1, [0])], [], mode="auto", schedule="concurrent")
    with pytest.raises(RuntimeError, match="unknown transfer mode"):
        kt.swap_batch([(1, [0])], [], mode="sideways")
    assert calls == []
