"""GPU parity of the local gather/scatter kernel (both copy engines) against the
reference's golden vectors and the C oracle; bit-exact throughout."""
import ctypes
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from lmpool_b200 import _capi
from lmpool_b200 import kv_transfer as kt
from oracle import c_oracle
from tests import kvgen

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
DEV = torch.device("cuda", 0)


@pytest.fixture(params=[1, 2], ids=["register", "bulk"])
def variant(request, require_gpu):
    lib = require_gpu
    old = _capi.Tuning()
    lib.kvx_get_tuning(ctypes.byref(old))
    lib.kvx_set_tuning(ctypes.byref(_capi.Tuning(variant=request.param)))
    yield request.param
    lib.kvx_set_tuning(ctypes.byref(old))
    kt.check_device_status(0)


def _bits_tensor(bits: np.ndarray, dtype) -> torch.Tensor:
    view = {2: torch.int16, 4: torch.int32}[torch.empty((), dtype=dtype).element_size()]
    return torch.from_numpy(bits.copy()).view(view).view(dtype)


def _same_bits(a: torch.Tensor, b: torch.Tensor) -> bool:
    a, b = a.detach().contiguous().cpu(), b.detach().contiguous().cpu()
    return a.shape == b.shape and torch.equal(a.view(torch.uint8), b.view(torch.uint8))


@pytest.mark.parametrize("case,dtype", [("c", torch.bfloat16), ("d", torch.float16)])
def test_pack_unpack_match_reference_golden(variant, case, dtype):
    z = np.load(GOLDEN / "pack_unpack.npz")
    src = _bits_tensor(z[f"{case}_src"], dtype).to(DEV)
    dst = _bits_tensor(z[f"{case}_dst_before"], dtype).to(DEV)
    L = src.shape[1]
    payload = kt._pack_all_layer_blocks(src, L, z[f"{case}_src_ids"].tolist())
    assert payload.is_contiguous()
    assert _same_bits(payload, _bits_tensor(z[f"{case}_payload"], dtype))
    kt._unpack_all_layer_blocks(payload, dst, z[f"{case}_dst_ids"].tolist())
    assert _same_bits(dst, _bits_tensor(z[f"{case}_dst_after"], dtype))
    kt.check_device_status(0)


def test_list_of_layer_views_matches_reference_golden(variant):
    z = np.load(GOLDEN / "pack_unpack.npz")
    big_src = _bits_tensor(z["e_src"], torch.bfloat16).to(DEV)
    big_dst = _bits_tensor(z["e_dst_before"], torch.bfloat16).to(DEV)
    L = big_src.shape[1]
    src_list = [(big_src[0, layer], big_src[1, layer]) for layer in range(L)]
    dst_list = [(big_dst[0, layer], big_dst[1, layer]) for layer in range(L)]
    payload = kt._pack_all_layer_blocks(src_list, L, z["e_src_ids"].tolist())
    assert _same_bits(payload, _bits_tensor(z["e_payload"], torch.bfloat16))
    kt._unpack_all_layer_blocks(payload, dst_list, z["e_dst_ids"].tolist())
    assert _same_bits(big_dst, _bits_tensor(z["e_dst_after"], torch.bfloat16))


def test_reference_unit_cases_on_gpu(variant):
    # tests/test_kv_transfer.py:66-79 and :82-102, float32 (24-byte chunks: narrow vector path)
    z = np.load(GOLDEN / "pack_unpack.npz")
    sk, sv = torch.from_numpy(z["a_source_k"]).to(DEV), torch.from_numpy(z["a_source_v"]).to(DEV)
    tk, tv = torch.zeros_like(sk), torch.zeros_like(sv)
    payload = kt._pack_layer_blocks(sk, sv, [3, 1])
    assert payload.is_contiguous() and torch.equal(payload.cpu(), torch.from_numpy(z["a_payload"]))
    kt._unpack_layer_blocks(payload, tk, tv, [0, 2])
    assert torch.equal(tk.cpu(), torch.from_numpy(z["a_target_k"]))
    assert torch.equal(tv.cpu(), torch.from_numpy(z["a_target_v"]))

    src = torch.from_numpy(z["b_source"]).to(DEV)  # [L, 2, N, ...]
    source = [(src[layer, 0], src[layer, 1]) for layer in range(2)]
    target = [(torch.zeros_like(k), torch.zeros_like(v)) for k, v in source]
    payload = kt._pack_all_layer_blocks(source, 2, [3, 1])
    assert payload.shape == (2, 2, 2, 3, 2, 1) and payload.is_contiguous()
    assert torch.equal(payload.cpu(), torch.from_numpy(z["b_payload"]))
    kt._unpack_all_layer_blocks(payload, target, [0, 2])
    got = torch.stack([torch.stack([k, v]) for k, v in target]).cpu()
    assert torch.equal(got, torch.from_numpy(z["b_target"]))


GEOMS = [
    # (shape [2, L, N, bs, H, D], dtype, B, seed)
    ((2, 28, 24, 256, 8, 128), torch.bfloat16, 8, 1),     # Qwen3-0.6B geometry, 512 KiB chunks
    ((2, 80, 40, 16, 8, 128), torch.bfloat16, 17, 2),     # 70B-like, 32 KiB chunks
    ((2, 3, 9, 5, 3, 7), torch.float32, 4, 3),            # 420-byte chunks: 4-byte vectors
    ((2, 2, 7, 3, 1, 3), torch.float16, 7, 4),            # 18-byte chunks: 2-byte vectors, B = N
    ((2, 1, 5, 1, 1, 1), torch.uint8, 3, 5),              # 1-byte chunks
]


@pytest.mark.parametrize("shape,dtype,B,seed", GEOMS)
def test_move_blocks_matches_oracle(variant, shape, dtype, B, seed):
    N = shape[2]
    if dtype == torch.uint8:
        g = torch.Generator().manual_seed(seed)
        src_cpu = torch.randint(0, 256, shape, generator=g, dtype=torch.uint8)
        dst_cpu = torch.randint(0, 256, shape, generator=g, dtype=torch.uint8)
    else:
        src_cpu = kvgen.seeded_cache(shape, seed, dtype)
        dst_cpu = kvgen.seeded_cache(shape, seed + 100, dtype)
    perm = kvgen.seeded_perm(N, seed)
    src_ids = perm[:B]
    dst_ids = kvgen.seeded_perm(N, seed + 7)[:B]
    src_ids[-1] = src_ids[0]  # a repeated source id is legal (index_select)
    src, dst = src_cpu.to(DEV), dst_cpu.to(DEV)
    out = kt.move_blocks(src, shape[1], src_ids, dst_ids, dst_kv_cache=dst, synchronize=True)
    assert out == dst_ids
    c_oracle.swap_planned(src_cpu, src_ids, dst_cpu, dst_ids, nthreads=4)
    assert _same_bits(dst, dst_cpu), "destination differs from the oracle (moved or untouched blocks)"
    assert _same_bits(src, src_cpu), "source cache was modified"


def test_move_within_one_cache_with_overlapping_ids(variant):
    shape = (2, 4, 12, 16, 2, 64)
    cpu = kvgen.seeded_cache(shape, 9)
    gpu = cpu.to(DEV)
    src_ids, dst_ids = [1, 2, 3, 4], [3, 4, 5, 6]   # overlap: reference semantics need the payload
    kt.move_blocks(gpu, 4, src_ids, dst_ids, synchronize=True)
    c_oracle.swap_planned(cpu, src_ids, cpu, dst_ids)
    assert _same_bits(gpu, cpu)


def test_move_within_one_cache_disjoint_ids_single_launch(variant):
    shape = (2, 5, 16, 32, 2, 64)
    cpu = kvgen.seeded_cache(shape, 12)
    gpu = cpu.to(DEV)
    perm = kvgen.seeded_perm(16, 12)
    src_ids, dst_ids = perm[:6], perm[6:12]
    kt.move_blocks(gpu, 5, src_ids, dst_ids, synchronize=True)
    c_oracle.swap_planned(cpu, src_ids, cpu, dst_ids)
    assert _same_bits(gpu, cpu)


def test_config1_geometry_matches_reference_digests(variant):
    """benchmark config 1 data, moved on the GPU: digests equal the reference's gloo swap_in."""
    rec = json.loads((GOLDEN / "swap_config1.json").read_text())
    src, dst, src_ids, dst_ids = kvgen.config1_inputs()
    src, dst = src.to(DEV), dst.to(DEV)
    kt.move_blocks(src, 28, src_ids, dst_ids, dst_kv_cache=dst, synchronize=True)
    assert kvgen.sha256_of(dst) == rec["dst_after_sha256"]
    assert kvgen.sha256_of(src) == rec["src_after_sha256"]


def test_duplicate_destination_ids_are_rejected(require_gpu):
    cache = torch.zeros(2, 1, 4, 2, 1, 8, device=DEV)
    with pytest.raises(RuntimeError, match="more than once"):
        kt.move_blocks(cache, 1, [0, 1], [2, 2])
    with pytest.raises(RuntimeError, match="outside"):
        kt.move_blocks(cache, 1, [0, 9], [2, 3])


def test_kernel_bounds_check_flags_and_skips_bad_ids(variant):
    """Ids that bypass host validation are caught by the kernel before any access."""
    lib = variant and _capi.lib()
    shape = (2, 2, 6, 4, 2, 16)
    src = kvgen.seeded_cache(shape, 31).to(DEV)
    dst = torch.zeros(shape, dtype=torch.bfloat16, device=DEV)
    from lmpool_b200.layout import affine_layout
    sl, dl = affine_layout(src, 2), affine_layout(dst, 2)
    src_ids = torch.tensor([1, 6, 2], dtype=torch.int64, device=DEV)     # 6 is out of range
    dst_ids = torch.tensor([0, 1, 7], dtype=torch.int64, device=DEV)     # 7 is out of range
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    sd, dd = sl.desc(), dl.desc()
    _capi.check(lib.kvx_move_blocks(0, ctypes.byref(sd), ctypes.byref(dd), ctypes.c_void_p(src_ids.data_ptr()),
                                    ctypes.c_void_p(dst_ids.data_ptr()), 3, ctypes.c_void_p(status.data_ptr()),
                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "move")
    torch.cuda.synchronize()
    bits = int(status.item())
    assert bits & _capi.DEV_BAD_SRC_ID and bits & _capi.DEV_BAD_DST_ID
    assert torch.equal(dst[:, :, 0], src[:, :, 1])          # the valid item moved
    assert dst[:, :, 1:].abs().sum().item() == 0             # nothing else was written


def test_full_config2_size_properties(variant):
    """benchmark config 2 at full size (L=28, N=2048, ~60 GB), B=512 fragmented ids:
    moved blocks equal their sources and every other block keeps its checksum."""
    free, _ = torch.cuda.mem_get_info()
    shape = (2, 28, 2048, 256, 8, 128)
    need = 2 * 28 * 2048 * 256 * 8 * 128 * 2
    if free < need + (8 << 30):
        pytest.skip("not enough device memory for the full config 2 cache")
    cache = torch.empty(shape, dtype=torch.bfloat16, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(0)
    cache.normal_(generator=g)
    perm = kvgen.seeded_perm(2048, 0)
    src_ids, dst_ids = perm[:512], perm[512:1024]

    def block_sums(t):
        # per (plane, layer, block) sum of the bf16 bit patterns, accumulated
        # in int64 one (plane, layer) slice at a time (bounded temporaries)
        out = torch.empty(2, 28, 2048, dtype=torch.int64, device=DEV)
        for kv in range(2):
            for layer in range(28):
                out[kv, layer] = t[kv, layer].view(torch.int16).view(2048, -1).sum(dim=-1, dtype=torch.int64)
        return out

    before = block_sums(cache)
    kt.move_blocks(cache, 28, src_ids, dst_ids, synchronize=True)
    after = block_sums(cache)
    untouched = torch.ones(2048, dtype=torch.bool)
    untouched[dst_ids] = False
    assert torch.equal(after[:, :, untouched.to(DEV)], before[:, :, untouched.to(DEV)])
    s = torch.tensor(src_ids, device=DEV)
    d = torch.tensor(dst_ids, device=DEV)
    assert torch.equal(after[:, :, d], before[:, :, s])
    for i in (0, 255, 511):   # spot-check whole blocks bit for bit
        assert torch.equal(cache[:, :, dst_ids[i]].view(torch.int16), cache[:, :, src_ids[i]].view(torch.int16))
    del cache
    torch.cuda.empty_cache()
