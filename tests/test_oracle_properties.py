"""Randomised agreement of the two oracle restatements (threaded C and plain
numpy) beyond the fixed golden cases: any geometry, element size, repeated
source ids, distinct targets, a move inside one cache with overlapping ids,
and store_kvcache with padding slots. Both are pinned to the reference's own
outputs by test_oracle_golden.py; this keeps them agreeing everywhere else."""
import numpy as np
import pytest
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import c_oracle, numpy_ref

DTYPES = [torch.uint8, torch.int16, torch.int32]


@st.composite
def moves(draw):
    L = draw(st.integers(1, 4))
    N = draw(st.integers(1, 12))
    bs, H, D = draw(st.integers(1, 5)), draw(st.integers(1, 3)), draw(st.integers(1, 9))
    dtype = draw(st.sampled_from(DTYPES))
    B = draw(st.integers(0, N))
    src_ids = draw(st.lists(st.integers(0, N - 1), min_size=B, max_size=B))
    dst_ids = draw(st.permutations(list(range(N))))[:B]
    same_cache = draw(st.booleans())
    threads = draw(st.sampled_from([1, 3]))
    seed = draw(st.integers(0, 2**31 - 1))
    return (2, L, N, bs, H, D), dtype, src_ids, dst_ids, same_cache, threads, seed


def _rand(shape, dtype, gen):
    info = torch.iinfo(dtype)
    return torch.randint(max(info.min, -(2**15)), min(info.max, 2**15 - 1) + 1, shape, generator=gen, dtype=torch.int64
                         ).to(dtype)


@settings(max_examples=80, deadline=None)
@given(moves())
def test_c_and_numpy_oracles_agree_on_any_planned_move(case):
    shape, dtype, src_ids, dst_ids, same_cache, threads, seed = case
    gen = torch.Generator().manual_seed(seed)
    src = _rand(shape, dtype, gen)
    dst = src if same_cache else _rand(shape, dtype, gen)
    src_np, dst_np = src.numpy().copy(), dst.numpy().copy()
    if same_cache:
        dst_np = src_np
    c_oracle.swap_planned(src, src_ids, dst, dst_ids, nthreads=threads)
    numpy_ref.swap_planned(src_np, src_ids, dst_np, dst_ids)
    assert np.array_equal(dst.numpy(), dst_np)
    if not same_cache:
        assert np.array_equal(src.numpy(), src_np), "source changed"


@settings(max_examples=40, deadline=None)
@given(moves())
def test_pack_then_unpack_to_the_same_ids_is_the_identity(case):
    shape, dtype, src_ids, _dst, _same, threads, seed = case
    ids = sorted(set(src_ids))
    cache = _rand(shape, dtype, torch.Generator().manual_seed(seed))
    before = cache.clone()
    payload = c_oracle.pack_all_layer_blocks(cache, ids, nthreads=threads)
    assert tuple(payload.shape) == (shape[1], 2, len(ids), *shape[3:])
    assert np.array_equal(payload.numpy(), numpy_ref.pack_all_layer_blocks(cache.numpy(), ids))
    if ids:
        c_oracle.unpack_all_layer_blocks(payload, cache, ids, nthreads=threads)
    assert torch.equal(cache, before)


@settings(max_examples=60, deadline=None)
@given(st.integers(0, 40), st.integers(1, 6), st.integers(1, 3), st.integers(1, 8),
       st.sampled_from([torch.int16, torch.int32]), st.floats(0.0, 0.6), st.integers(0, 2**31 - 1))
def test_c_and_numpy_store_kvcache_agree(T, N, H, D, dtype, pad, seed):
    bs = 4
    gen = torch.Generator().manual_seed(seed)
    key, value = _rand((T, H, D), dtype, gen), _rand((T, H, D), dtype, gen)
    kc, vc = _rand((N, bs, H, D), dtype, gen), _rand((N, bs, H, D), dtype, gen)
    T_valid = min(T, N * bs)
    slots = torch.full((T,), -1, dtype=torch.int64)
    slots[:T_valid] = torch.randperm(N * bs, generator=gen)[:T_valid]
    slots[torch.rand(T, generator=gen) < pad] = -1
    kn, vn = kc.numpy().copy(), vc.numpy().copy()
    assert c_oracle.store_kvcache(key, value, kc, vc, slots, bs) == 0
    numpy_ref.store_kvcache(key.numpy(), value.numpy(), kn, vn, slots.numpy(), bs)
    assert np.array_equal(kc.numpy(), kn) and np.array_equal(vc.numpy(), vn)


def test_numpy_oracle_refuses_what_the_reference_refuses():
    cache = np.zeros((2, 1, 4, 1, 1, 2), dtype=np.uint16)
    with pytest.raises(RuntimeError, match="mismatched"):
        numpy_ref.swap_planned(cache, [0, 1], cache.copy(), [2])
    with pytest.raises(RuntimeError, match="distinct"):
        numpy_ref.swap_planned(cache, [0, 1], cache.copy(), [2, 2])
