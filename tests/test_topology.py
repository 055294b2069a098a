"""NVLink pair detection (drop-in for global_block_manager.py:38-98), on CPU
with a fake NVML and a fake peer-access query, and on the GPU box against
the driver. The reference's own cases (tests/test_global_block_manager.py:
427-448: two NVLink GPUs give [(0, 1)]; a failing tool gives []) are kept."""
import pytest

from lmpool_b200.topology import detect_nvlink_pairs
from tests.conftest import device_count


class FakeNVML:
    NVML_P2P_CAPS_INDEX_NVLINK = 2
    NVML_P2P_STATUS_OK = 0

    def __init__(self, nvlinked: set[frozenset[str]], fail: str = ""):
        self.nvlinked = nvlinked
        self.fail = fail
        self.calls = []

    def nvmlInit(self):
        self.calls.append("init")
        if self.fail == "init":
            raise RuntimeError("NVML Shared Library Not Found")

    def nvmlShutdown(self):
        self.calls.append("shutdown")

    def nvmlDeviceGetHandleByPciBusId(self, bus_id):
        return bus_id

    def nvmlDeviceGetP2PStatus(self, a, b, index):
        assert index == self.NVML_P2P_CAPS_INDEX_NVLINK
        if self.fail == "query":
            raise RuntimeError("not supported")
        return self.NVML_P2P_STATUS_OK if frozenset((a, b)) in self.nvlinked else 5


BUS = [f"00000000:{0x18 + 0x10 * i:02X}:00.0" for i in range(8)]


def test_two_nvlinked_gpus_give_one_pair_like_the_reference():
    nvml = FakeNVML({frozenset(BUS[:2])})
    assert detect_nvlink_pairs(2, nvml=nvml, bus_ids=BUS[:2]) == [(0, 1)]
    assert nvml.calls == ["init", "shutdown"]


def test_pairs_follow_the_visible_order_and_world_size():
    # CUDA_VISIBLE_DEVICES=5,2,7: logical 0,1,2 are physical 5,2,7; only 2-7 share NVLink
    visible = [BUS[5], BUS[2], BUS[7]]
    nvml = FakeNVML({frozenset((BUS[2], BUS[7]))})
    assert detect_nvlink_pairs(3, nvml=nvml, bus_ids=visible) == [(1, 2)]
    assert detect_nvlink_pairs(2, nvml=nvml, bus_ids=visible) == []
    everything = FakeNVML({frozenset((a, b)) for a in BUS for b in BUS if a != b})
    assert detect_nvlink_pairs(8, nvml=everything, bus_ids=BUS) == [(a, b) for a in range(8) for b in range(a + 1, 8)]


@pytest.mark.parametrize("fail", ["init", "query"])
def test_without_nvml_the_cuda_peer_query_decides(fail):
    nvml = FakeNVML(set(), fail=fail)
    both_ways = {(0, 1), (1, 0), (2, 3), (3, 2), (1, 2)}   # 1->2 only one way: not a pair
    got = detect_nvlink_pairs(4, nvml=nvml, bus_ids=BUS[:4], can_access=lambda a, b: (a, b) in both_ways)
    assert got == [(0, 1), (2, 3)]


def test_failures_and_small_worlds_give_an_empty_list():
    def broken(a, b):
        raise RuntimeError("driver gone")

    assert detect_nvlink_pairs(2, nvml=FakeNVML(set(), fail="init"), bus_ids=BUS[:2], can_access=broken) == []
    assert detect_nvlink_pairs(1, nvml=FakeNVML(set()), bus_ids=BUS[:4]) == []
    assert detect_nvlink_pairs(4, nvml=FakeNVML(set()), bus_ids=[]) == []


@pytest.mark.gpu
@pytest.mark.skipif(device_count() < 2, reason="needs 2 GPUs")
def test_b200_box_reports_nvlink_between_visible_gpus(require_gpu):
    n = device_count()
    pairs = detect_nvlink_pairs(n)
    # an HGX B200 box: every pair of GPUs meets at the NVSwitch
    assert pairs == [(a, b) for a in range(n) for b in range(a + 1, n)]
    # the CUDA peer-access fallback agrees
    assert detect_nvlink_pairs(n, nvml=FakeNVML(set(), fail="init")) == pairs
