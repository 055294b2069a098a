"""Host logic of the drop-in: layout normalisation, pair normalisation,
reference helper parity and error behaviour. CPU only; no kernel runs."""
import pytest
import torch

from lmpool_b200 import kv_transfer as kt
from lmpool_b200.layout import affine_layout, cache_layouts, get_layer_kv, payload_layout


# -- reference tests/test_kv_transfer.py:42-63, same assertions ---------------

def test_kv_transfer_helpers_are_stable():
    kv_cache = torch.zeros(2, 4, 2, 1, 1)
    view = kt._allocate_empty_block(kv_cache, 2)
    assert view.shape == (2, 2, 1, 1)
    assert kt._compute_tag(3, 4, True) != kt._compute_tag(3, 4, False)
    assert kt._compute_tag(3, 4, True) != kt._compute_tag(4, 4, True)


def test_transfer_pairs_are_normalized_and_filtered():
    assert kt._normalize_transfer_pairs([(1, 0), (0, 1), (2, 2), (3, 8)], 4) == [(0, 1)]
    assert kt._normalize_transfer_pairs([(3, 2), (0, 1), (-1, 2)], 4) == [(0, 1), (2, 3)]


def test_get_layer_kv_accepts_model_runner_cache_layout():
    k0 = torch.zeros(4, 2, 1, 1)
    v0 = torch.ones(4, 2, 1, 1)
    k1 = torch.full((4, 2, 1, 1), 2.0)
    v1 = torch.full((4, 2, 1, 1), 3.0)
    layer_k, layer_v = kt._get_layer_kv([(k0, v0), (k1, v1)], 1)
    assert layer_k is k1 and layer_v is v1


def test_get_layer_kv_rejects_unknown_layouts():
    with pytest.raises(RuntimeError, match="Unsupported kv_cache layout"):
        get_layer_kv(torch.zeros(3, 3), 0)
    with pytest.raises(RuntimeError, match="empty kv_cache"):
        get_layer_kv([], 0)


# -- layouts -----------------------------------------------------------------

def test_six_d_tensor_is_one_affine_layout():
    t = torch.zeros(2, 3, 5, 4, 2, 8, dtype=torch.bfloat16)
    (lay,) = cache_layouts(t, 3)
    e = 2
    assert lay.base == t.data_ptr()
    assert lay.kv_stride == t.stride(0) * e
    assert lay.layer_stride == t.stride(1) * e
    assert lay.block_stride == t.stride(2) * e
    assert lay.chunk_bytes == 4 * 2 * 8 * e
    assert (lay.num_blocks, lay.num_layers) == (5, 3)
    # block (kv=1, layer=2, block=4) offset matches element indexing
    assert lay.base + lay.block_offset(1, 2, 4) == t[1, 2, 4].data_ptr()


def test_model_runner_list_of_views_is_affine():
    t = torch.zeros(2, 4, 6, 2, 1, 8)
    views = [(t[0, layer], t[1, layer]) for layer in range(4)]
    lay = affine_layout(views, 4)
    (ref,) = cache_layouts(t, 4)
    assert (lay.base, lay.kv_stride, lay.layer_stride, lay.block_stride) == (
        ref.base, ref.kv_stride, ref.layer_stride, ref.block_stride)


def test_separate_tensors_fall_back_to_per_layer_layouts():
    layers = [(torch.zeros(4, 2, 1, 8), torch.zeros(4, 2, 1, 8)) for _ in range(3)]
    lays = cache_layouts(layers, 3)
    assert len(lays) == 3 and all(l.num_layers == 1 for l in lays)
    with pytest.raises(RuntimeError, match="constant stride"):
        affine_layout(layers, 3)


def test_five_d_single_layer_maps_every_layer_to_itself():
    t = torch.zeros(2, 5, 4, 2, 8)
    (lay,) = cache_layouts(t, 3)
    assert lay.layer_stride == 0 and lay.num_layers == 3


def test_non_contiguous_block_is_rejected():
    t = torch.zeros(2, 1, 4, 8, 2, 16)[..., ::2]
    with pytest.raises(RuntimeError, match="contiguous"):
        cache_layouts(t, 1)


def test_payload_layout_matches_reference_payload_indexing():
    L, B, shape = 3, 4, (2, 1, 8)
    p = torch.zeros(L, 2, B, *shape, dtype=torch.float16)
    lay = payload_layout(L, B, shape, p.dtype, p.device, p.data_ptr())
    assert lay.base + lay.block_offset(1, 2, 3) == p[2, 1, 3].data_ptr()
    assert lay.base + lay.block_offset(0, 1, 0) == p[1, 0, 0].data_ptr()


# -- error behaviour (no GPU needed: raised before any launch) ---------------

def test_cpu_tensors_are_refused_not_silently_handled(kvx_lib):
    cache = torch.zeros(2, 1, 4, 2, 1, 8)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        kt._pack_all_layer_blocks(cache, 1, [0])
    payload = torch.zeros(1, 2, 1, 2, 1, 8)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        kt._unpack_all_layer_blocks(payload, cache, [0])


def test_empty_plans_are_no_ops_like_the_reference():
    cache = torch.zeros(2, 2, 4, 2, 1, 8)
    payload = kt._pack_all_layer_blocks(cache, 2, [])
    assert payload.shape == (2, 2, 0, 2, 1, 8)
    kt._unpack_all_layer_blocks(torch.zeros(2, 2, 0, 2, 1, 8), cache, [])
    assert kt._pack_layer_blocks(cache[0, 0], cache[1, 0], []).shape == (2, 0, 2, 1, 8)


def test_payload_count_mismatch_raises_like_the_reference():
    cache = torch.zeros(2, 2, 4, 2, 1, 8)
    with pytest.raises(RuntimeError, match="does not match destination blocks"):
        kt._unpack_all_layer_blocks(torch.zeros(2, 2, 3, 2, 1, 8), cache, [0, 1])
    with pytest.raises(RuntimeError, match="does not match destination block count"):
        kt._unpack_layer_blocks(torch.zeros(2, 3, 2, 1, 8), cache[0, 0], cache[1, 0], [0])


def test_move_blocks_count_mismatch_raises():
    cache = torch.zeros(2, 1, 4, 2, 1, 8)
    with pytest.raises(RuntimeError, match="destination ids"):
        kt.move_blocks(cache, 1, [0, 1], [2])


def test_prewarm_without_process_group_returns_empty():
    assert kt.prewarm_p2p_pairs([(0, 1)]) == []


def test_drop_in_module_exposes_the_reference_names_and_ours():
    # every name of src/lmpool/engine/kv_transfer.py, plus this package's additions
    reference = ["_normalize_transfer_pairs", "_pair_group", "prewarm_p2p_pairs", "_allocate_empty_block",
                 "_compute_tag", "_get_layer_kv", "_pack_layer_blocks", "_unpack_layer_blocks", "_empty_layer_payload",
                 "_pack_all_layer_blocks", "_empty_all_layer_payload", "_unpack_all_layer_blocks", "_send_block_list",
                 "_recv_block_list", "swap_out", "swap_in", "request_free_blocks", "respond_free_blocks", "_P2P_GROUPS"]
    ours = ["register_kv_cache", "move_blocks", "swap_batch", "check_device_status", "shutdown", "transfer_mode"]
    missing = [n for n in reference + ours if not hasattr(kt, n)]
    assert not missing, missing


def test_transfer_mode_defaults_to_pull_and_validates(monkeypatch):
    monkeypatch.delenv("LMPOOL_B200_KV_MODE", raising=False)
    assert kt.transfer_mode() == "pull"
    monkeypatch.setenv("LMPOOL_B200_KV_MODE", "push")
    assert kt.transfer_mode() == "push"
    monkeypatch.setenv("LMPOOL_B200_KV_MODE", "sideways")
    with pytest.raises(RuntimeError, match="pull"):
        kt.transfer_mode()
