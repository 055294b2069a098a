"""GPU parity of store_kvcache against the reference Triton kernel's golden
outputs and the C oracle; bit-exact."""
from pathlib import Path

import numpy as np
import pytest
import torch

from lmpool_b200 import _capi
from lmpool_b200 import kv_transfer as kt
from lmpool_b200.attention import store_kvcache, store_kvcache_layers
from oracle import c_oracle
from tests import kvgen

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
DEV = torch.device("cuda", 0)


def _bits_tensor(bits: np.ndarray, dtype) -> torch.Tensor:
    view = {2: torch.int16, 4: torch.int32}[torch.empty((), dtype=dtype).element_size()]
    return torch.from_numpy(bits.copy()).view(view).view(dtype)


def _same_bits(a, b) -> bool:
    a, b = a.detach().contiguous().cpu(), b.detach().contiguous().cpu()
    return a.shape == b.shape and torch.equal(a.view(torch.uint8), b.view(torch.uint8))


@pytest.mark.parametrize("case", ["f32", "bf16", "h8"])
def test_matches_reference_triton_kernel_outputs(require_gpu, case):
    z = np.load(GOLDEN / "store_kvcache.npz")
    T, H, D, bs, N = z[f"{case}_dims"].tolist()
    dtype = torch.float32 if case == "f32" else torch.bfloat16
    key = _bits_tensor(z[f"{case}_key"], dtype).to(DEV)
    value = _bits_tensor(z[f"{case}_value"], dtype).to(DEV)
    kc = _bits_tensor(z[f"{case}_kc_before"], dtype).to(DEV)
    vc = _bits_tensor(z[f"{case}_vc_before"], dtype).to(DEV)
    slots = torch.from_numpy(z[f"{case}_slots"]).to(DEV)
    store_kvcache(key, value, kc, vc, slots, bs)
    kt.check_device_status(0)
    assert _same_bits(kc, _bits_tensor(z[f"{case}_kc_after"], dtype))
    assert _same_bits(vc, _bits_tensor(z[f"{case}_vc_after"], dtype))


def test_config5_geometry_matches_oracle(require_gpu):
    """benchmark config 5: T=256 tokens, H=8, D=128, block_size=16, ~10% padding slots (N shrunk)."""
    T, H, D, bs, N = 256, 8, 128, 16, 4096
    key_c = kvgen.seeded_cache((T, H, D), 70)
    value_c = kvgen.seeded_cache((T, H, D), 71)
    kc_c = kvgen.seeded_cache((N, bs, H, D), 72)
    vc_c = kvgen.seeded_cache((N, bs, H, D), 73)
    slots_c = kvgen.slot_mapping(T, N * bs, 74, skip_fraction=0.1)
    key, value, kc, vc, slots = (t.to(DEV) for t in (key_c, value_c, kc_c, vc_c, slots_c))
    store_kvcache(key, value, kc, vc, slots, bs)
    kt.check_device_status(0)
    assert c_oracle.store_kvcache(key_c, value_c, kc_c, vc_c, slots_c, bs) == 0
    assert _same_bits(kc, kc_c) and _same_bits(vc, vc_c)


def test_non_contiguous_inputs_and_strided_rows(require_gpu):
    T, H, D, bs, N = 40, 4, 32, 8, 16
    big = kvgen.seeded_cache((T, 2, H, D), 80)
    key_c, value_c = big[:, 0], big[:, 1]              # token stride 2*H*D: not contiguous
    kc_c = kvgen.seeded_cache((N, bs, H, D), 81)
    vc_c = kvgen.seeded_cache((N, bs, H, D), 82)
    slots_c = kvgen.slot_mapping(T, N * bs, 83)
    key, value = big.to(DEV)[:, 0], big.to(DEV)[:, 1]
    kc, vc, slots = kc_c.to(DEV), vc_c.to(DEV), slots_c.to(DEV)
    store_kvcache(key, value, kc, vc, slots, bs)
    kt.check_device_status(0)
    c_oracle.store_kvcache(key_c, value_c, kc_c, vc_c, slots_c, bs)
    assert _same_bits(kc, kc_c) and _same_bits(vc, vc_c)


def test_all_layers_in_one_launch_matches_per_layer_oracle(require_gpu):
    L, T, H, D, bs, N = 80, 64, 8, 128, 16, 64
    keys_c = kvgen.seeded_cache((L, T, H, D), 90)
    values_c = kvgen.seeded_cache((L, T, H, D), 91)
    cache_c = kvgen.seeded_cache((2, L, N, bs, H, D), 92)
    slots_c = kvgen.slot_mapping(T, N * bs, 93)
    keys, values, cache, slots = (t.to(DEV) for t in (keys_c, values_c, cache_c, slots_c))
    store_kvcache_layers(keys, values, cache, slots, bs)
    kt.check_device_status(0)
    for layer in range(L):
        c_oracle.store_kvcache(keys_c[layer], values_c[layer], cache_c[0, layer], cache_c[1, layer], slots_c, bs)
    assert _same_bits(cache, cache_c)


def test_out_of_range_slots_are_flagged_and_skipped(require_gpu):
    T, H, D, bs, N = 4, 1, 8, 2, 3
    key = torch.ones(T, H, D, device=DEV)
    kc = torch.zeros(N, bs, H, D, device=DEV)
    vc = torch.zeros(N, bs, H, D, device=DEV)
    slots = torch.tensor([0, 6, -5, -1], dtype=torch.int64, device=DEV)
    store_kvcache(key, key, kc, vc, slots, bs)
    with pytest.raises(_capi.KvxError, match="slot_mapping"):
        kt.check_device_status(0)
    assert kc.view(N * bs, -1)[0].eq(1).all() and kc.view(N * bs, -1)[1:].abs().sum() == 0


@pytest.fixture(params=[1, 2], ids=["pdl", "no_pdl"])
def store_launch(request, require_gpu):
    """Run the test with store_kvcache launched with programmatic dependent
    launch (the default) and without it."""
    import ctypes

    lib = require_gpu
    old = _capi.Tuning()
    lib.kvx_get_tuning(ctypes.byref(old))
    t = _capi.Tuning()
    ctypes.memmove(ctypes.byref(t), ctypes.byref(old), ctypes.sizeof(t))
    t.store_pdl = request.param
    assert lib.kvx_set_tuning(ctypes.byref(t)) == 0
    yield request.param
    lib.kvx_set_tuning(ctypes.byref(old))


def test_store_sees_rows_the_kernel_before_it_wrote(store_launch):
    """Each step writes new K/V rows with a kernel and stores them at once,
    eagerly and captured in a graph (as a model layer does): the store reads
    the new rows every time, with or without programmatic dependent launch."""
    T, H, D, bs, N, L = 64, 8, 128, 16, 96, 6
    kc = torch.zeros(L, N, bs, H, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    key = torch.zeros(L, T, H, D, dtype=torch.bfloat16, device=DEV)
    value = torch.zeros_like(key)
    src_k = kvgen.seeded_cache((L, T, H, D), 130).to(DEV)
    src_v = kvgen.seeded_cache((L, T, H, D), 131).to(DEV)
    slots = kvgen.slot_mapping(T, N * bs, 132, skip_fraction=0.1).to(DEV)
    scale = torch.ones((), dtype=torch.bfloat16, device=DEV)

    def step():
        for layer in range(L):
            torch.mul(src_k[layer], scale, out=key[layer])        # a kernel writes the rows ...
            torch.mul(src_v[layer], scale, out=value[layer])
            store_kvcache(key[layer], value[layer], kc[layer], vc[layer], slots, bs)   # ... stored right after

    def expected():
        kc_c = torch.zeros(L, N, bs, H, D, dtype=torch.bfloat16)
        vc_c = torch.zeros_like(kc_c)
        for layer in range(L):
            c_oracle.store_kvcache((src_k[layer] * scale).cpu(), (src_v[layer] * scale).cpu(), kc_c[layer],
                                   vc_c[layer], slots.cpu(), bs)
        return kc_c, vc_c

    for rnd in range(5):
        scale.fill_(float(rnd + 1))
        step()
    torch.cuda.synchronize()
    kt.check_device_status(0)
    kc_c, vc_c = expected()
    assert _same_bits(kc, kc_c) and _same_bits(vc, vc_c)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for rnd in range(5):
        scale.fill_(float(rnd + 7))
        graph.replay()
        torch.cuda.synchronize()
        kc_c, vc_c = expected()
        assert _same_bits(kc, kc_c) and _same_bits(vc, vc_c)
    kt.check_device_status(0)


def test_captured_in_a_cuda_graph(require_gpu):
    """The decode path captures store_kvcache (model_runner.py:630-683): no sync, no allocation."""
    T, H, D, bs, N = 32, 8, 128, 16, 64
    key = kvgen.seeded_cache((T, H, D), 95).to(DEV)
    value = kvgen.seeded_cache((T, H, D), 96).to(DEV)
    kc = torch.zeros(N, bs, H, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    slots = torch.full((T,), -1, dtype=torch.int64, device=DEV)
    store_kvcache(key, value, kc, vc, slots, bs)     # warm-up outside capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        store_kvcache(key, value, kc, vc, slots, bs)
    new_slots = kvgen.slot_mapping(T, N * bs, 97).to(DEV)
    slots.copy_(new_slots)
    graph.replay()
    torch.cuda.synchronize()
    kt.check_device_status(0)
    kc_c, vc_c = torch.zeros(N, bs, H, D, dtype=torch.bfloat16), torch.zeros(N, bs, H, D, dtype=torch.bfloat16)
    c_oracle.store_kvcache(key.cpu(), value.cpu(), kc_c, vc_c, new_slots.cpu(), bs)
    assert _same_bits(kc, kc_c) and _same_bits(vc, vc_c)


def test_argument_errors(require_gpu):
    key = torch.zeros(2, 1, 8, device=DEV)
    kc = torch.zeros(2, 2, 1, 8, device=DEV)
    with pytest.raises(AssertionError):
        store_kvcache(key, key, kc, kc, torch.zeros(3, dtype=torch.int64, device=DEV), 2)
    with pytest.raises(TypeError):
        store_kvcache(key, key, kc, kc, torch.zeros(2, dtype=torch.int32, device=DEV), 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        store_kvcache(key.cpu(), key.cpu(), kc.cpu(), kc.cpu(), torch.zeros(2, dtype=torch.int64), 2)
