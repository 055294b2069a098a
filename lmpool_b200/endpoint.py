"""Per-GPU transfer endpoint: mailbox, peer mappings and the pair protocol.

One :class:`TransferEndpoint` exists per (process, GPU). It owns this rank's
mailbox (a small device region other ranks write into over NVLink), the
mappings of peers' KV caches and mailboxes (CUDA IPC for other processes,
plain peer pointers inside one process), and the completion tokens of every
directed pair. It replaces the per-pair NCCL communicators of
``prewarm_p2p_pairs`` (src/lmpool/engine/kv_transfer.py:40-119) and the
``dist.send``/``dist.recv`` of ``swap_in`` (kv_transfer.py:463-470).

Protocol of one transfer ``src -> dst`` (B blocks), push mode:

=================================  ==========================================
destination (execute_swap_in)      source (execute_swap_out)
=================================  ==========================================
token = next token for src
publish: ids -> src mailbox,
  count, arm = token               wait_armed: arm > last consumed
                                     (bounded), count == B, go = token
wait_done: flag == token           push: src blocks -> dst cache over NVLink;
  (bounded)                          last CTA: flag = token (release, sys)
stream sync, status check          stream sync, status check
=================================  ==========================================

Pull mode (the default of ``swap_in``):

=================================  ==========================================
destination (execute_swap_in)      source (execute_swap_out)
=================================  ==========================================
token = next token for src
request: count | PULL, arm = token
  -> src mailbox                   grant: arm > last consumed (bounded),
                                     count == B | PULL, then flag = token
                                     (release, sys) on the source's stream,
                                     after every earlier write there
wait_done: flag == token (bounded)
pull: src blocks over NVLink ->
  own blocks, only if flag is
  still token; last CTA:
  pulled = token (| FAIL)          [wait_pulled: pulled > last consumed]
stream sync, status check          [stream sync, status check]
=================================  ==========================================

Tokens are issued by the destination and only grow, so a late or repeated
completion can never satisfy a newer transfer, and a source that missed a
transfer simply consumes the newest arm. All waits are bounded and end with
an error status, never a hang or a trap.
"""
from __future__ import annotations

import ctypes
import logging
import os
import threading
from dataclasses import dataclass, field

import torch

from . import _capi
from .layout import CacheLayout

logger = logging.getLogger(__name__)

DEFAULT_TIMEOUT_S = float(os.environ.get("LMPOOL_B200_KV_TIMEOUT_S", "120"))
MAX_TARGETS_PER_LAUNCH = 8


def _dtype_from_name(name: str) -> torch.dtype:
    dt = getattr(torch, str(name).split(".")[-1], None)
    return dt if isinstance(dt, torch.dtype) else torch.uint8


def timeout_ns(seconds: float | None) -> int:
    s = DEFAULT_TIMEOUT_S if seconds is None else float(seconds)
    return max(1, int(s * 1e9))


@dataclass
class PeerRecord:
    """What a rank publishes about itself to the others (plain data)."""

    rank: int
    pid: int
    hostname: str
    device: int
    mailbox_handle: bytes
    mailbox_offset: int
    mailbox_ptr: int
    mailbox_peers: int
    mailbox_max_blocks: int
    cache_handle: bytes | None = None
    cache_offset: int = 0
    cache_ptr: int = 0
    cache_geometry: dict | None = None
    extra: dict = field(default_factory=dict)


@dataclass
class PeerLink:
    """This process's view of one peer: its mailbox and cache, mapped here."""

    peer: int
    mailbox: _capi.Mailbox
    cache: CacheLayout | None
    closers: list = field(default_factory=list)  # IPC handles to release on close
    poisoned: str | None = None


def pair_round(a: int, b: int, world_size: int) -> int:
    """Round of the pair {a, b} in a round-robin tournament over
    ``world_size`` ranks (the circle method): rank m-1 (m = world_size
    rounded up to even) meets rank r in round r; any other two ranks meet in
    the round r with a + b = 2r (mod m-1). Each of the m-1 rounds is a
    perfect matching, and the value is the same for (a, b) and (b, a)."""
    a, b = int(a), int(b)
    if a == b or not (0 <= a < world_size and 0 <= b < world_size):
        raise RuntimeError(f"no round for the pair ({a}, {b}) among {world_size} ranks")
    m = world_size + (world_size % 2)
    if a == m - 1 or b == m - 1:
        return b if a == m - 1 else a
    return ((a + b) * (m // 2)) % (m - 1)


class TransferEndpoint:
    """Mailbox, peer links and pair tokens of one rank on one GPU."""

    def __init__(self, rank: int, world_size: int, device: int, max_blocks: int):
        if world_size <= 0 or not (0 <= rank < world_size):
            raise RuntimeError(f"bad rank {rank} for world size {world_size}")
        self.rank = int(rank)
        self.world_size = int(world_size)
        self.device = int(device)
        self.lib = _capi.lib()
        mb = _capi.Mailbox()
        _capi.check(self.lib.kvx_mailbox_create(self.device, self.world_size, int(max_blocks), ctypes.byref(mb)),
                    "kvx_mailbox_create")
        self.mailbox = mb
        self.cache: CacheLayout | None = None
        self._cache_ref = None
        self.links: dict[int, PeerLink] = {}
        self.tokens_issued: dict[int, int] = {}
        self._lock = threading.Lock()
        self._ipc_maps: dict[bytes, list] = {}   # handle -> [base address, references]
        # word 0: this endpoint's per-call status (zeroed per transfer); read
        # back through a pinned word, one copy and one stream sync per check
        self.status = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", self.device))
        self.status_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._status_host_np = self.status_host.numpy()
        self.status_clean = True    # the device word is zero and nothing enqueued since
        self.mode = "pull"          # pair transfer mode used by exchange(); the same on every rank
        self.closed = False

    # -- local cache ---------------------------------------------------------
    def set_cache(self, layout: CacheLayout, keepalive=None) -> None:
        if layout.device.type != "cuda" or layout.device.index != self.device:
            raise RuntimeError(f"cache lives on {layout.device}, endpoint is on cuda:{self.device}")
        if layout.num_blocks > self.mailbox.max_blocks:
            raise RuntimeError(
                f"cache has {layout.num_blocks} blocks, mailbox holds {self.mailbox.max_blocks}: "
                "create the endpoint with max_blocks >= num_blocks"
            )
        self.cache = layout
        self._cache_ref = keepalive

    # -- records and links ---------------------------------------------------
    def export_record(self, hostname: str = "") -> PeerRecord:
        handle = ctypes.create_string_buffer(64)
        off = ctypes.c_uint64(0)
        _capi.check(self.lib.kvx_ipc_export(self.device, ctypes.c_void_p(self.mailbox.base), handle, ctypes.byref(off)),
                    "kvx_ipc_export(mailbox)")
        rec = PeerRecord(rank=self.rank, pid=os.getpid(), hostname=hostname, device=self.device,
                         mailbox_handle=handle.raw, mailbox_offset=off.value, mailbox_ptr=self.mailbox.base,
                         mailbox_peers=self.mailbox.max_peers, mailbox_max_blocks=self.mailbox.max_blocks)
        if self.cache is not None:
            ch = ctypes.create_string_buffer(64)
            coff = ctypes.c_uint64(0)
            _capi.check(self.lib.kvx_ipc_export(self.device, ctypes.c_void_p(self.cache.base), ch, ctypes.byref(coff)),
                        "kvx_ipc_export(kv cache)")
            rec.cache_handle = ch.raw
            rec.cache_offset = coff.value
            rec.cache_ptr = self.cache.base
            rec.cache_geometry = self.cache.geometry()
        return rec

    def export_buffer(self, ptr: int) -> tuple[bytes, int]:
        handle = ctypes.create_string_buffer(64)
        off = ctypes.c_uint64(0)
        _capi.check(self.lib.kvx_ipc_export(self.device, ctypes.c_void_p(ptr), handle, ctypes.byref(off)),
                    "kvx_ipc_export")
        return handle.raw, off.value

    def map_buffer(self, rec_pid: int, rec_device: int, handle: bytes, offset: int, ptr: int,
                   closers: list | None) -> int:
        """Address of a peer buffer usable from this GPU.

        Other processes' buffers are opened through CUDA IPC once per
        allocation (two buffers of one allocator segment share a handle) and
        reference-counted; ``closers`` receives the handle to release.
        """
        if rec_pid == os.getpid():
            if rec_device != self.device:
                _capi.check(self.lib.kvx_enable_peer_access(self.device, rec_device), "kvx_enable_peer_access")
            return int(ptr)
        key = bytes(handle)
        entry = self._ipc_maps.get(key)
        if entry is None:
            out = ctypes.c_uint64(0)
            _capi.check(self.lib.kvx_ipc_open(self.device, key, 0, ctypes.byref(out)), "kvx_ipc_open")
            entry = [int(out.value), 0]
            self._ipc_maps[key] = entry
        entry[1] += 1
        if closers is not None:
            closers.append(key)
        return entry[0] + int(offset)

    def unmap_buffer(self, key: bytes) -> None:
        entry = self._ipc_maps.get(key)
        if entry is None:
            return
        entry[1] -= 1
        if entry[1] <= 0:
            del self._ipc_maps[key]
            _capi.check(self.lib.kvx_ipc_close(self.device, entry[0], 0), "kvx_ipc_close")

    def link(self, rec: PeerRecord) -> PeerLink:
        """Map a peer's mailbox and KV cache (idempotent)."""
        with self._lock:
            if rec.rank in self.links:
                return self.links[rec.rank]
            if rec.rank == self.rank:
                raise RuntimeError("a rank does not link to itself")
            if rec.mailbox_peers != self.world_size:
                raise RuntimeError(f"peer {rec.rank} mailbox is for {rec.mailbox_peers} ranks, expected "
                                   f"{self.world_size}")
            if rec.pid != os.getpid():
                ok = ctypes.c_int32(0)
                _capi.check(self.lib.kvx_can_access_peer(self.device, rec.device, ctypes.byref(ok)),
                            "kvx_can_access_peer")
                if not ok.value:
                    raise RuntimeError(f"cuda:{self.device} cannot access peer cuda:{rec.device} over NVLink/P2P")
            closers: list = []
            mb_ptr = self.map_buffer(rec.pid, rec.device, rec.mailbox_handle, rec.mailbox_offset, rec.mailbox_ptr,
                                     closers)
            mailbox = _capi.Mailbox(base=mb_ptr, max_peers=rec.mailbox_peers, reserved=0,
                                    max_blocks=rec.mailbox_max_blocks)
            cache = None
            if rec.cache_geometry is not None:
                base = self.map_buffer(rec.pid, rec.device, rec.cache_handle, rec.cache_offset, rec.cache_ptr,
                                       closers)
                g = rec.cache_geometry
                cache = CacheLayout(base=base, kv_stride=g["kv_stride"], layer_stride=g["layer_stride"],
                                    block_stride=g["block_stride"], num_blocks=g["num_blocks"],
                                    chunk_bytes=g["chunk_bytes"], num_layers=g["num_layers"],
                                    dtype=_dtype_from_name(g.get("dtype", "torch.uint8")),
                                    device=torch.device("cuda", rec.device), block_shape=tuple(g["block_shape"]))
            link = PeerLink(peer=rec.rank, mailbox=mailbox, cache=cache, closers=closers)
            self.links[rec.rank] = link
            return link

    def get_link(self, peer: int) -> PeerLink:
        link = self.links.get(int(peer))
        if link is None:
            raise RuntimeError(
                f"rank {self.rank} has no mapping of rank {peer}: call prewarm_p2p_pairs "
                "(every rank, after register_kv_cache) before transferring"
            )
        if link.poisoned:
            raise RuntimeError(f"pair ({self.rank}, {peer}) is disabled after an earlier failure: {link.poisoned}")
        return link

    def next_token(self, src_rank: int) -> int:
        with self._lock:
            t = self.tokens_issued.get(src_rank, 0) + 1
            self.tokens_issued[src_rank] = t
            return t

    # -- protocol steps (enqueue only) ----------------------------------------
    def publish(self, link: PeerLink, dst_ids: torch.Tensor, num_ids: int, token: int, stream) -> None:
        self.status_clean = False
        _capi.check(self.lib.kvx_pair_publish(self.device, ctypes.byref(link.mailbox), self.rank,
                                              ctypes.c_void_p(dst_ids.data_ptr() if num_ids else 0), num_ids, token,
                                              ctypes.c_void_p(_capi.stream_handle(stream))),
                    "kvx_pair_publish")

    def wait_done(self, src_rank: int, token: int, timeout_s: float | None, stream) -> None:
        self.status_clean = False
        _capi.check(self.lib.kvx_pair_wait_done(self.device, ctypes.byref(self.mailbox), src_rank, token,
                                                timeout_ns(timeout_s), ctypes.c_void_p(self.status.data_ptr()),
                                                ctypes.c_void_p(_capi.stream_handle(stream))),
                    "kvx_pair_wait_done")

    def request(self, link: PeerLink, num_ids: int, token: int, stream) -> None:
        """Pull: ask the source (link.peer) to grant ``num_ids`` blocks under ``token``."""
        self.status_clean = False
        _capi.check(self.lib.kvx_pair_request(self.device, ctypes.byref(link.mailbox), self.rank, num_ids, token,
                                              ctypes.c_void_p(_capi.stream_handle(stream))),
                    "kvx_pair_request")

    def grant(self, link: PeerLink, num_ids: int, timeout_s: float | None, stream, status_ptr: int | None = None) -> None:
        """Pull: answer the destination's request once this stream reaches here."""
        if status_ptr is None:
            self.status_clean = False
            status_ptr = self.status.data_ptr()
        _capi.check(self.lib.kvx_pair_grant(self.device, ctypes.byref(self.mailbox), ctypes.byref(link.mailbox),
                                            self.rank, link.peer, num_ids, timeout_ns(timeout_s),
                                            ctypes.c_void_p(status_ptr), ctypes.c_void_p(_capi.stream_handle(stream))),
                    "kvx_pair_grant")

    # -- grants whose outcome is read later (source returns once enqueued) ---
    ASYNC_SLOTS = 32

    def grant_deferred(self, link: PeerLink, num_ids: int, timeout_s: float | None, stream, what: str) -> None:
        """Enqueue a grant without waiting for it or for the destination's read.

        The grant reports into a status word of its own; a copy of that word
        to pinned host memory and an event follow it on ``stream``, and
        :meth:`poll_deferred` reads the outcome once the event has completed,
        so nothing here or later blocks on it. A failed grant disables the
        pair (its next use raises); the destination side of the same
        transfer fails on its own bounded wait.
        """
        self.poll_deferred()
        if not hasattr(self, "_async_dev"):
            dev = torch.device("cuda", self.device)
            self._async_dev = torch.zeros(self.ASYNC_SLOTS, dtype=torch.int32, device=dev)
            self._async_host = torch.zeros(self.ASYNC_SLOTS, dtype=torch.int32).pin_memory()
            self._async_np = self._async_host.numpy()
            self._async_free = list(range(self.ASYNC_SLOTS))
            self._async_pending: list = []
        if not self._async_free:            # all slots in flight: wait for the oldest
            self._async_pending[0][1].synchronize()
            self.poll_deferred()
        i = self._async_free.pop()
        word = self._async_dev[i:i + 1]
        with torch.cuda.stream(stream):
            word.zero_()
            self.grant(link, num_ids, timeout_s, stream, status_ptr=word.data_ptr())
            self._async_host[i:i + 1].copy_(word, non_blocking=True)
            event = torch.cuda.Event()
            event.record(stream)
        self._async_pending.append((i, event, what, link.peer))

    def poll_deferred(self, wait: bool = False) -> None:
        """Read the outcome of deferred grants that have completed (all of
        them when ``wait``); a failure is logged and disables its pair."""
        pending = getattr(self, "_async_pending", None)
        if not pending:
            return
        keep = []
        for i, event, what, peer in pending:
            if wait:
                event.synchronize()
            elif not event.query():
                keep.append((i, event, what, peer))
                continue
            bits = int(self._async_np[i])
            self._async_free.append(i)
            if bits:
                msg = f"{what}: {_capi.describe_device_status(bits)}"
                logger.error("deferred grant failed on rank %d: %s", self.rank, msg)
                link = self.links.get(peer)
                if link is not None:
                    link.poisoned = msg
        self._async_pending = keep

    def reset_pair(self, peer: int, stream) -> None:
        """Forget every token of the pair (this rank, ``peer``): zero the pair's
        words in this rank's mailbox and restart this side's token count.
        Both ranks do it, with nothing of the pair in flight, before either
        transfers again (prewarm runs it on every rank, between barriers)."""
        _capi.check(self.lib.kvx_mailbox_reset_peer(self.device, ctypes.byref(self.mailbox), int(peer),
                                                    ctypes.c_void_p(_capi.stream_handle(stream))),
                    "kvx_mailbox_reset_peer")
        with self._lock:
            self.tokens_issued.pop(int(peer), None)
        link = self.links.get(int(peer))
        if link is not None:
            link.poisoned = None

    def wait_armed(self, link: PeerLink, num_ids: int, timeout_s: float | None, stream) -> None:
        self.status_clean = False
        _capi.check(self.lib.kvx_pair_wait_armed(self.device, ctypes.byref(self.mailbox), ctypes.byref(link.mailbox),
                                                 self.rank, link.peer, num_ids, timeout_ns(timeout_s),
                                                 ctypes.c_void_p(self.status.data_ptr()),
                                                 ctypes.c_void_p(_capi.stream_handle(stream))),
                    "kvx_pair_wait_armed")

    def push(self, src: CacheLayout, targets: list[tuple[PeerLink, CacheLayout, torch.Tensor, int]], stream) -> None:
        """One launch per group of up to 8 targets: (link, peer layout, src ids, count)."""
        self.status_clean = False
        for start in range(0, len(targets), MAX_TARGETS_PER_LAUNCH):
            group = targets[start:start + MAX_TARGETS_PER_LAUNCH]
            arr = (_capi.PushTarget * len(group))()
            for k, (link, peer_layout, ids, n) in enumerate(group):
                arr[k].dst = peer_layout.desc()
                arr[k].dst_mailbox = link.mailbox
                arr[k].src_ids_dev = ids.data_ptr() if n else 0
                arr[k].num_ids = n
                arr[k].dst_rank = link.peer
                arr[k].reserved = 0
            src_desc = src.desc()
            _capi.check(self.lib.kvx_pair_push(self.device, ctypes.byref(src_desc), ctypes.byref(self.mailbox),
                                               self.rank, arr, len(group), ctypes.c_void_p(self.status.data_ptr()),
                                               ctypes.c_void_p(_capi.stream_handle(stream))),
                        "kvx_pair_push")

    def pull(self, local: CacheLayout, sources: list[tuple], stream) -> None:
        """Destination-driven copy: one launch per group of up to 8 sources,
        each (link, peer layout, src ids, dst ids, count, token)."""
        self.status_clean = False
        dst_desc = local.desc()
        for start in range(0, len(sources), MAX_TARGETS_PER_LAUNCH):
            group = sources[start:start + MAX_TARGETS_PER_LAUNCH]
            arr = (_capi.PullSource * len(group))()
            for k, (link, peer_layout, sids, dids, n, token) in enumerate(group):
                arr[k].src = peer_layout.desc()
                arr[k].src_mailbox = link.mailbox
                arr[k].src_ids_dev = sids.data_ptr() if n else 0
                arr[k].dst_ids_dev = dids.data_ptr() if n else 0
                arr[k].num_ids = n
                arr[k].token = token
                arr[k].src_rank = link.peer
                arr[k].reserved = 0
            _capi.check(self.lib.kvx_pair_pull(self.device, ctypes.byref(dst_desc), ctypes.byref(self.mailbox),
                                               self.rank, arr, len(group), ctypes.c_void_p(self.status.data_ptr()),
                                               ctypes.c_void_p(_capi.stream_handle(stream))),
                        "kvx_pair_pull")

    def wait_pulled(self, dst_rank: int, timeout_s: float | None, stream) -> None:
        self.status_clean = False
        _capi.check(self.lib.kvx_pair_wait_pulled(self.device, ctypes.byref(self.mailbox), dst_rank,
                                                  timeout_ns(timeout_s), ctypes.c_void_p(self.status.data_ptr()),
                                                  ctypes.c_void_p(_capi.stream_handle(stream))),
                    "kvx_pair_wait_pulled")

    def exchange(self, mode: str, local: CacheLayout, outgoing: list[tuple], incoming: list[tuple],
                 timeout_s: float | None, stream, peer_layouts: dict | None = None,
                 wait_pulled: bool = True) -> None:
        """Enqueue every transfer of this rank (no host wait).

        ``outgoing`` = [(dst_rank, src ids, count)] of blocks this rank gives;
        ``incoming`` = [(src_rank, src ids, dst ids, count)] of blocks it
        receives (src ids are used in pull mode only). ``peer_layouts`` maps a
        rank to the peer layout to read or write (default: the peer's cache).
        Push: arms for every incoming transfer first, then one push launch
        for all outgoing ones, then the completion waits. Pull: requests for
        every incoming transfer first, then the grants of this rank's
        outgoing blocks, then the waits for the incoming grants and one pull
        launch for all incoming transfers, then (``wait_pulled``) the waits
        for the peers that read this rank's blocks. Either order leaves no
        wait depending on a later launch of any rank.
        """
        self.status_clean = False
        layouts = peer_layouts or {}
        if mode == "push":
            tokens = []
            for src_rank, _sids, dids, n in incoming:
                token = self.next_token(src_rank)
                self.publish(self.get_link(src_rank), dids, n, token, stream)
                tokens.append((src_rank, token))
            targets = []
            for dst_rank, sids, n in outgoing:
                link = self.get_link(dst_rank)
                self.wait_armed(link, n, timeout_s, stream)
                targets.append((link, layouts.get(dst_rank, link.cache), sids, n))
            if targets:
                self.push(local, targets, stream)
            for src_rank, token in tokens:
                self.wait_done(src_rank, token, timeout_s, stream)
        elif mode == "pull":
            sources = []
            for src_rank, sids, dids, n in incoming:
                link = self.get_link(src_rank)
                token = self.next_token(src_rank)
                self.request(link, n, token, stream)
                sources.append((link, layouts.get(src_rank, link.cache), sids, dids, n, token))
            for dst_rank, _sids, n in outgoing:
                self.grant(self.get_link(dst_rank), n, timeout_s, stream)
            for link, _layout, _sids, _dids, _n, token in sources:
                self.wait_done(link.peer, token, timeout_s, stream)
            if sources:
                self.pull(local, sources, stream)
            if wait_pulled:
                for dst_rank, _sids, _n in outgoing:
                    self.wait_pulled(dst_rank, timeout_s, stream)
        else:
            raise RuntimeError(f"unknown transfer mode {mode!r}: expected 'pull' or 'push'")

    def exchange_rotated(self, mode: str, local: CacheLayout, outgoing: list[tuple], incoming: list[tuple],
                         timeout_s: float | None, stream, peer_layouts: dict | None = None,
                         wait_pulled: bool = True) -> None:
        """The transfers of ``exchange`` in rounds of disjoint pairs.

        Rounds follow a round-robin tournament over the ranks
        (:func:`pair_round`): each round pairs every rank with at most one
        partner, and both directions between two ranks fall in the same
        round. So at any moment every GPU sends to one peer and receives from
        that peer (the traffic of disjoint pairs exchanging both ways)
        instead of serving all peers at once, and a pair that sends both ways
        is never split across rounds. Each rank enqueues its rounds in
        increasing order and a round only waits on that round's steps of its
        one partner, so no wait depends on a later round. Every rank of a call
        must use this schedule.

        ``mode="auto"`` picks the mode per round: push when this rank and its
        partner send each other blocks in that round (writes cost fewer wire
        bytes than reads when both directions are busy), pull when the round
        is one-way (reads cost fewer). Both ranks of a round see the same
        pair of lists, so they pick the same mode.
        """
        if mode not in ("push", "pull", "auto"):
            raise RuntimeError(f"unknown transfer mode {mode!r}: expected 'pull', 'push' or 'auto'")
        world = self.world_size
        rounds: dict[int, tuple[list, list]] = {}
        for item in outgoing:
            rounds.setdefault(pair_round(self.rank, item[0], world), ([], []))[0].append(item)
        for item in incoming:
            rounds.setdefault(pair_round(item[0], self.rank, world), ([], []))[1].append(item)
        for j in sorted(rounds):
            out, inc = rounds[j]
            round_mode = mode
            if mode == "auto":
                two_way = {o[0] for o in out} & {i[0] for i in inc}
                round_mode = "push" if two_way else "pull"
            self.exchange(round_mode, local, out, inc, timeout_s, stream, peer_layouts, wait_pulled)

    def read_done(self, src_rank: int) -> int:
        out = ctypes.c_uint64(0)
        _capi.check(self.lib.kvx_mailbox_read_done(self.device, ctypes.byref(self.mailbox), src_rank,
                                                   ctypes.byref(out)), "kvx_mailbox_read_done")
        return out.value

    def reset_status(self, stream) -> None:
        """Zero the status word on ``stream`` before a transfer, unless the
        last check read zero and nothing has been enqueued since."""
        if not self.status_clean:
            with torch.cuda.stream(stream):
                self.status.zero_()

    def check_status(self, stream, what: str, peers=()) -> None:
        if stream == torch.cuda.current_stream(self.device):
            self.status_host.copy_(self.status, non_blocking=True)
        else:
            with torch.cuda.stream(stream):
                self.status_host.copy_(self.status, non_blocking=True)
        stream.synchronize()
        bits = int(self._status_host_np[0])
        if not bits:
            self.status_clean = True
        else:
            if bits & (_capi.DEV_TIMEOUT | _capi.DEV_PIPE_TIMEOUT):
                # A peer that is merely late may still write into blocks this
                # rank is about to give back; refuse further use of the pair.
                for p in peers:
                    if p in self.links:
                        self.links[p].poisoned = f"{what}: {_capi.describe_device_status(bits)}"
            raise _capi.KvxError(f"{what} failed on rank {self.rank}: {_capi.describe_device_status(bits)}",
                                 status=_capi.KVX_EINVAL, device_bits=bits)

    def close_links(self) -> None:
        """Release every peer mapping (the peers' memory stays theirs)."""
        for link in self.links.values():
            for key in link.closers:
                try:
                    self.unmap_buffer(key)
                except Exception as exc:  # noqa: BLE001 - best effort at shutdown
                    logger.warning("closing peer mapping failed: %s", exc)
            link.closers = []
        self.links.clear()

    def close(self) -> None:
        if self.closed:
            return
        try:
            self.poll_deferred(wait=True)
        except Exception as exc:  # noqa: BLE001 - best effort at shutdown
            logger.warning("reading deferred grants failed: %s", exc)
        for link in self.links.values():
            for key in link.closers:
                try:
                    self.unmap_buffer(key)
                except Exception as exc:  # noqa: BLE001 - best effort at shutdown
                    logger.warning("closing peer mapping failed: %s", exc)
        self.links.clear()
        try:
            _capi.check(self.lib.kvx_mailbox_destroy(self.device, ctypes.byref(self.mailbox)), "kvx_mailbox_destroy")
        finally:
            self.closed = True
