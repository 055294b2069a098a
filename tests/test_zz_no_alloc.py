"""kvx_pair_push_noalloc: the push for callers that cannot call cudaMalloc.

Some callers of this library cannot allocate device memory: a serving process
whose GPU memory is already taken (LMPool gives its KV cache the configured
share of all free memory), a plugin whose host program forbids it to allocate
device memory, or a host whose own allocator owns all device memory. The
allocation-free push keeps the kernel's scratch (per-destination CTA-completion counters) in a fixed
array inside the library, so such a caller needs nothing allocated for it.

This test calls it through the C ABI and checks its output against the
existing kvx_pair_push on the same transfer, bit for bit, twice in a row
(the second call reuses the array the first one left behind). One GPU hosts
a source rank and two destination ranks; every step runs in order on one
stream, so each bounded wait is satisfied by a kernel that already finished.
"""
import ctypes

import pytest
import torch

from lmpool_b200 import _capi
from lmpool_b200.endpoint import TransferEndpoint
from lmpool_b200.layout import affine_layout
from oracle import c_oracle
from tests import kvgen

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _same_bits(a, b) -> bool:
    a, b = a.detach().contiguous().cpu(), b.detach().contiguous().cpu()
    return a.shape == b.shape and torch.equal(a.view(torch.uint8), b.view(torch.uint8))


def test_noalloc_push_matches_existing_push_on_two_calls(require_gpu):
    lib = require_gpu
    shape = (2, 8, 24, 256, 8, 128)
    N = shape[2]
    src_cpu = kvgen.seeded_cache(shape, 301)
    ref_cpu = kvgen.seeded_cache(shape, 302)
    src = src_cpu.to(DEV)
    dst_existing = ref_cpu.to(DEV)
    dst_noalloc = ref_cpu.to(DEV)
    ep0 = TransferEndpoint(0, 3, 0, N)
    ep1 = TransferEndpoint(1, 3, 0, N)
    ep2 = TransferEndpoint(2, 3, 0, N)
    ep0.set_cache(affine_layout(src, shape[1]), src)
    ep1.set_cache(affine_layout(dst_existing, shape[1]), dst_existing)
    ep2.set_cache(affine_layout(dst_noalloc, shape[1]), dst_noalloc)
    l01 = ep0.link(ep1.export_record())
    l02 = ep0.link(ep2.export_record())
    l10 = ep1.link(ep0.export_record())
    l20 = ep2.link(ep0.export_record())
    s = torch.cuda.current_stream(DEV)
    try:
        for call in range(2):
            src_ids = kvgen.seeded_perm(N, 310 + call)[:7]
            dst_ids = kvgen.seeded_perm(N, 320 + call)[:7]
            src_t = torch.tensor(src_ids, dtype=torch.int64, device=DEV)
            dst_t = torch.tensor(dst_ids, dtype=torch.int64, device=DEV)
            for ep in (ep0, ep1, ep2):
                ep.status.zero_()
            t1 = ep1.next_token(0)
            t2 = ep2.next_token(0)
            ep1.publish(l10, dst_t, 7, t1, s)
            ep2.publish(l20, dst_t, 7, t2, s)
            ep0.wait_armed(l01, 7, 5.0, s)
            ep0.wait_armed(l02, 7, 5.0, s)
            ep0.push(ep0.cache, [(l01, l01.cache, src_t, 7)], s)          # existing entry point
            target = _capi.PushTarget(dst=l02.cache.desc(), dst_mailbox=l02.mailbox, src_ids_dev=src_t.data_ptr(),
                                      num_ids=7, dst_rank=2, reserved=0)
            src_desc = ep0.cache.desc()
            _capi.check(lib.kvx_pair_push_noalloc(0, ctypes.byref(src_desc), ctypes.byref(ep0.mailbox), 0,
                                                  ctypes.byref(target), 1, ctypes.c_void_p(ep0.status.data_ptr()),
                                                  ctypes.c_void_p(s.cuda_stream)),
                        "kvx_pair_push_noalloc")
            ep1.wait_done(0, t1, 5.0, s)
            ep2.wait_done(0, t2, 5.0, s)
            ep0.check_status(s, "source")
            ep1.check_status(s, "destination (existing push)")
            ep2.check_status(s, "destination (allocation-free push)")
            assert _same_bits(dst_noalloc, dst_existing), f"call {call}: outputs differ"
            c_oracle.swap_planned(src_cpu, src_ids, ref_cpu, dst_ids, nthreads=4)
            assert _same_bits(dst_existing, ref_cpu), f"call {call}: existing push differs from the oracle"
    finally:
        for ep in (ep0, ep1, ep2):
            ep.close_links()
        for ep in (ep0, ep1, ep2):
            ep.close()


def test_noalloc_push_rejects_ranks_beyond_its_array(kvx_lib):
    """Checked before any device work, so this needs no GPU."""
    desc = _capi.CacheDesc(base=1 << 30, kv_stride=4096, layer_stride=8192, block_stride=16, num_blocks=4,
                           chunk_bytes=16, num_layers=1, reserved=0)
    mb = _capi.Mailbox(base=1 << 31, max_peers=128, reserved=0, max_blocks=4)
    target = _capi.PushTarget(dst=desc, dst_mailbox=mb, src_ids_dev=1 << 32, num_ids=1,
                              dst_rank=_capi.NOALLOC_MAX_PEERS, reserved=0)
    status = ctypes.c_int32(0)
    rc = kvx_lib.kvx_pair_push_noalloc(0, ctypes.byref(desc), ctypes.byref(mb), 0, ctypes.byref(target), 1,
                                       ctypes.byref(status), None)
    assert rc == _capi.KVX_EINVAL
    assert b"beyond the 64 ranks" in kvx_lib.kvx_last_error()
