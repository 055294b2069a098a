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
    return ep, calls


def test_push_arms_everything_before_any_wait():
    ep, calls = _endpoint(0, 4)
    ep.exchange("push", "local", [(1, "i1", 5), (2, "i2", 0)], [(1, "s1", "d1", 3), (3, "s3", "d3", 4)], 1.0, None)
    kinds = [c[0] for c in calls]
    assert kinds == ["publish", "publish", "wait_armed", "wait_armed", "push", "wait_done", "wait_done"]
    assert calls[0] == ("publish", 1, 3, 1) and calls[1] == ("publish", 3, 4, 1)
    assert calls[4] == ("push", [(1, "cache1", 5), (2, "cache2", 0)])
    assert calls[5] == ("wait_done", 1, 1) and calls[6] == ("wait_done", 3, 1)


def test_pull_reads_everything_before_any_wait():
    ep, calls = _endpoint(2, 4)
    ep.exchange("pull", "local", [(0, "i0", 5)], [(1, "s1", "d1", 3), (3, "s3", "d3", 0)], 1.0, None,
                peer_layouts={3: "payload3"})
    assert [c[0] for c in calls] == ["pull", "wait_pulled"]
    assert calls[0] == ("pull", [(1, "cache1", 3, 1), (3, "payload3", 0, 1)])
    assert calls[1] == ("wait_pulled", 0)


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
