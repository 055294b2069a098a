"""ModelRunner boundary on CPU: the mixin forwards to ``swap_in`` exactly as
LMPool's wrappers do (model_runner.py:747-806; the reference pins this in
tests/test_model_runner.py:218-246), counts bytes like kv_transfer_bytes
(model_runner.py:808-820) and collects caches like _get_kv_cache (:822-833)."""
import pytest
import torch

from lmpool_b200 import kv_transfer
from lmpool_b200.model_runner import B200KVTransferMixin


class _Layer(torch.nn.Module):
    def __init__(self, k=None, v=None):
        super().__init__()
        self.k_cache, self.v_cache = k, v


class _Runner(B200KVTransferMixin):
    def __init__(self, rank, layers, config):
        self.rank = rank
        self.block_size = 16
        self.config = config
        self.model = torch.nn.ModuleList(layers)


def _runner(rank=0, L=2, config=None):
    layers = [_Layer(torch.zeros(4, 16, 2, 8, dtype=torch.bfloat16), torch.zeros(4, 16, 2, 8, dtype=torch.bfloat16))
              for _ in range(L)]
    return _Runner(rank, layers, config or {"num_layers": L, "num_kv_heads": 2, "head_dim": 8})


def test_execute_swap_methods_forward_to_swap_in(monkeypatch):
    calls = []

    def fake_swap_in(**kwargs):
        calls.append(kwargs)
        return [9, 10]

    monkeypatch.setattr(kv_transfer, "swap_in", fake_swap_in)
    runner = _runner(rank=0)
    assert runner.execute_swap_out([1, 2], target_gpu=1) == [9, 10]
    assert runner.execute_swap_in(remote_gpu=1, remote_blocks=[3, 4], local_target_blocks=[5, 6]) == [9, 10]
    out, inn = calls
    # the source is the remote side of the destination's swap_in
    assert (out["remote_gpu"], out["remote_blocks"], out["local_gpu"]) == (0, [1, 2], 1)
    assert "local_target_blocks" not in out and out["negotiate_blocks"] is False
    assert (inn["remote_gpu"], inn["remote_blocks"], inn["local_gpu"]) == (1, [3, 4], 0)
    assert inn["local_target_blocks"] == [5, 6] and inn["negotiate_blocks"] is False
    for c in calls:
        assert (c["num_layers"], c["block_size"], c["num_kv_heads"], c["head_dim"]) == (2, 16, 2, 8)
        assert len(c["kv_cache"]) == 2 and all(len(kv) == 2 for kv in c["kv_cache"])


def test_head_dim_falls_back_to_hidden_size_over_heads(monkeypatch):
    seen = {}
    monkeypatch.setattr(kv_transfer, "swap_in", lambda **kw: seen.update(kw) or [])
    runner = _runner(config={"num_layers": 2, "num_kv_heads": 2, "hidden_size": 64, "num_heads": 8})
    runner.execute_swap_out([0], target_gpu=1)
    assert seen["head_dim"] == 8


def test_kv_transfer_bytes_and_cache_collection():
    runner = _runner(L=3, config={"num_layers": 3, "num_kv_heads": 2, "head_dim": 8})
    # n * L * (bs*H*D*itemsize) * 2
    assert runner.kv_transfer_bytes(5) == 5 * 3 * (16 * 2 * 8 * 2) * 2
    assert runner.kv_transfer_bytes(0) == 0
    runner.model.append(_Layer(torch.zeros(0), torch.zeros(0)))   # empty caches are skipped
    runner.model.append(_Layer())                                   # so are layers without them
    assert len(runner._get_kv_cache()) == 3
    empty = _Runner(0, [_Layer()], {"num_layers": 1})
    with pytest.raises(RuntimeError, match="Cannot find k_cache/v_cache"):
        empty._get_kv_cache()
