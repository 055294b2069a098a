"""Pin the CPU oracle (C and numpy restatements) to the reference's own outputs.

The fixtures in tests/golden/ were produced by LMPool's code
(tests/golden/make_golden.py): pack/unpack helpers, swap_in over two gloo
ranks, and the Triton store_kvcache under Triton's CPU interpreter.
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import c_oracle, numpy_ref
from tests import kvgen

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def pu():
    return np.load(GOLDEN / "pack_unpack.npz")


def _as_tensor(bits: np.ndarray, dtype) -> torch.Tensor:
    view = {2: torch.int16, 4: torch.int32}[torch.empty((), dtype=dtype).element_size()]
    return torch.from_numpy(bits.copy()).view(view).view(dtype)


def test_numpy_oracle_reference_case_a(pu):
    # tests/test_kv_transfer.py:66-79 (per-layer, arange float32)
    cache = np.stack([pu["a_source_k"], pu["a_source_v"]])[:, None]  # [2, 1, N, ...]
    payload = numpy_ref.pack_all_layer_blocks(cache, pu["a_src_ids"])
    assert np.array_equal(payload[0], pu["a_payload"])
    target = np.zeros_like(cache)
    numpy_ref.unpack_all_layer_blocks(payload, target, pu["a_dst_ids"])
    assert np.array_equal(target[0, 0], pu["a_target_k"])
    assert np.array_equal(target[1, 0], pu["a_target_v"])


def test_numpy_oracle_reference_case_b(pu):
    # tests/test_kv_transfer.py:82-102 (two layers, payload (2, 2, 2, 3, 2, 1))
    src = pu["b_source"].transpose(1, 0, 2, 3, 4, 5)  # [L, 2, ...] -> [2, L, ...]
    payload = numpy_ref.pack_all_layer_blocks(src, pu["b_src_ids"])
    assert payload.shape == (2, 2, 2, 3, 2, 1)
    assert np.array_equal(payload, pu["b_payload"])
    target = np.zeros_like(src)
    numpy_ref.unpack_all_layer_blocks(payload, target, pu["b_dst_ids"])
    assert np.array_equal(target, pu["b_target"].transpose(1, 0, 2, 3, 4, 5))


@pytest.mark.parametrize("case,dtype", [("c", torch.bfloat16), ("d", torch.float16), ("e", torch.bfloat16)])
def test_numpy_oracle_seeded_cases(pu, case, dtype):
    src = pu[f"{case}_src"]
    dst = pu[f"{case}_dst_before"].copy()
    payload = numpy_ref.pack_all_layer_blocks(src, pu[f"{case}_src_ids"])
    assert np.array_equal(payload, pu[f"{case}_payload"])
    numpy_ref.unpack_all_layer_blocks(payload, dst, pu[f"{case}_dst_ids"])
    assert np.array_equal(dst, pu[f"{case}_dst_after"])


@pytest.mark.parametrize("case,dtype", [("c", torch.bfloat16), ("d", torch.float16), ("e", torch.bfloat16)])
@pytest.mark.parametrize("threads", [1, 3])
def test_c_oracle_seeded_cases(pu, case, dtype, threads):
    src = _as_tensor(pu[f"{case}_src"], dtype)
    dst = _as_tensor(pu[f"{case}_dst_before"], dtype)
    payload = c_oracle.pack_all_layer_blocks(src, pu[f"{case}_src_ids"].tolist(), nthreads=threads)
    assert torch.equal(payload.view(torch.int16), _as_tensor(pu[f"{case}_payload"], dtype).view(torch.int16))
    c_oracle.unpack_all_layer_blocks(payload, dst, pu[f"{case}_dst_ids"].tolist(), nthreads=threads)
    assert torch.equal(dst.view(torch.int16), _as_tensor(pu[f"{case}_dst_after"], dtype).view(torch.int16))


def test_c_oracle_swap_small_matches_reference_gloo_run():
    z = np.load(GOLDEN / "swap_small.npz")
    src = torch.from_numpy(z["rank0_before"].copy())
    dst = torch.from_numpy(z["rank1_before"].copy())
    c_oracle.swap_planned(src, z["src_ids"].tolist(), dst, z["dst_ids"].tolist(), nthreads=2)
    assert torch.equal(src, torch.from_numpy(z["rank0_after"]))
    assert torch.equal(dst, torch.from_numpy(z["rank1_after"]))
    assert z["returned0"].tolist() == z["src_ids"].tolist()
    assert z["returned1"].tolist() == z["dst_ids"].tolist()


def test_c_oracle_rejects_duplicate_destinations_and_bad_ids():
    cache = torch.zeros(2, 1, 4, 2, 1, 1)
    payload = torch.ones(1, 2, 2, 2, 1, 1)
    with pytest.raises(RuntimeError):
        c_oracle.unpack_all_layer_blocks(payload, cache, [1, 1])
    with pytest.raises(RuntimeError):
        c_oracle.pack_all_layer_blocks(cache, [0, 4])
    with pytest.raises(RuntimeError):
        c_oracle.swap_planned(cache, [0, 1], cache.clone(), [2])


def test_c_oracle_config1_matches_reference_digests():
    """benchmark config 1: the reference's gloo swap_in digests, reproduced by the C oracle."""
    rec = json.loads((GOLDEN / "swap_config1.json").read_text())
    src, dst, src_ids, dst_ids = kvgen.config1_inputs()
    assert src_ids == rec["src_ids"] and dst_ids == rec["dst_ids"]
    assert kvgen.sha256_of(src) == rec["src_before_sha256"]
    assert kvgen.sha256_of(dst) == rec["dst_before_sha256"]
    c_oracle.swap_planned(src, src_ids, dst, dst_ids, nthreads=c_oracle.default_threads())
    assert kvgen.sha256_of(src) == rec["src_after_sha256"]
    assert kvgen.sha256_of(dst) == rec["dst_after_sha256"]


@pytest.mark.parametrize("case", ["f32", "bf16", "h8"])
def test_store_kvcache_oracles_match_reference_triton_kernel(case):
    z = np.load(GOLDEN / "store_kvcache.npz")
    T, H, D, bs, N = z[f"{case}_dims"].tolist()
    dtype = torch.float32 if case == "f32" else torch.bfloat16
    key = _as_tensor(z[f"{case}_key"], dtype)
    value = _as_tensor(z[f"{case}_value"], dtype)
    kc = _as_tensor(z[f"{case}_kc_before"], dtype)
    vc = _as_tensor(z[f"{case}_vc_before"], dtype)
    slots = torch.from_numpy(z[f"{case}_slots"])
    assert (slots == -1).any()
    # numpy restatement on raw bits
    kcn, vcn = z[f"{case}_kc_before"].copy(), z[f"{case}_vc_before"].copy()
    numpy_ref.store_kvcache(z[f"{case}_key"], z[f"{case}_value"], kcn, vcn, z[f"{case}_slots"], bs)
    assert np.array_equal(kcn, z[f"{case}_kc_after"]) and np.array_equal(vcn, z[f"{case}_vc_after"])
    # C restatement
    bad = c_oracle.store_kvcache(key, value, kc, vc, slots, bs)
    assert bad == 0
    ival = torch.int32 if dtype == torch.float32 else torch.int16
    assert torch.equal(kc.view(ival), _as_tensor(z[f"{case}_kc_after"], dtype).view(ival))
    assert torch.equal(vc.view(ival), _as_tensor(z[f"{case}_vc_after"], dtype).view(ival))


def test_c_oracle_store_kvcache_counts_out_of_range_slots():
    key = torch.ones(3, 1, 4)
    kc = torch.zeros(2, 2, 1, 4)
    vc = torch.zeros(2, 2, 1, 4)
    bad = c_oracle.store_kvcache(key, key, kc, vc, torch.tensor([0, 4, -2]), 2)
    assert bad == 2
    assert torch.equal(kc.view(4, 4)[0], torch.ones(4)) and kc.view(4, 4)[1:].abs().sum() == 0
