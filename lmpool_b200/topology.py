"""NVLink pair detection that asks the driver instead of parsing ``nvidia-smi``.

Drop-in for ``detect_nvlink_pairs_from_nvidia_smi(world_size)``
(src/lmpool/engine/global_block_manager.py:38-98), which GlobalBlockManager
calls when it is given no pairs (global_block_manager.py:139-141). Same
contract: pairs ``(a, b)`` of logical GPU indices with ``a < b < world_size``,
in this process's device order, sorted, and an empty list whenever the
topology cannot be determined.

Each pair of visible devices is checked with NVML's NVLink peer-to-peer
status (``nvmlDeviceGetP2PStatus`` with the NVLink capability). Devices are
matched to NVML handles by PCI bus id, so the pairs are in CUDA's logical
order even when ``CUDA_VISIBLE_DEVICES`` selects or reorders GPUs (the text
parser reads nvidia-smi's physical numbering). Without NVML the CUDA
peer-access query of ``kvx_can_access_peer`` is used instead; it also counts
PCIe peer pairs. On an NVSwitch box (HGX B200) every pair is an NVLink pair,
as nvidia-smi's ``NV18`` cells also say.

Only read-only queries are made: no GPU setting is changed.
"""
from __future__ import annotations

import ctypes
import logging
from typing import Callable, List, Optional, Sequence, Tuple

logger = logging.getLogger(__name__)


def _visible_pci_bus_ids() -> list[str]:
    import torch

    if not torch.cuda.is_available():
        return []
    ids = []
    for i in range(torch.cuda.device_count()):
        p = torch.cuda.get_device_properties(i)
        ids.append(f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0")
    return ids


def _nvml_pairs(nvml, bus_ids: Sequence[str]) -> list[tuple[int, int]]:
    nvml.nvmlInit()
    try:
        handles = [nvml.nvmlDeviceGetHandleByPciBusId(b) for b in bus_ids]
        pairs = []
        for a in range(len(handles)):
            for b in range(a + 1, len(handles)):
                status = nvml.nvmlDeviceGetP2PStatus(handles[a], handles[b], nvml.NVML_P2P_CAPS_INDEX_NVLINK)
                if status == nvml.NVML_P2P_STATUS_OK:
                    pairs.append((a, b))
        return pairs
    finally:
        nvml.nvmlShutdown()


def _kvx_can_access(device: int, peer: int) -> bool:
    from . import _capi

    ok = ctypes.c_int32(0)
    _capi.check(_capi.lib().kvx_can_access_peer(device, peer, ctypes.byref(ok)), "kvx_can_access_peer")
    return bool(ok.value)


def detect_nvlink_pairs(world_size: int, *, nvml=None, bus_ids: Optional[Sequence[str]] = None,
                        can_access: Optional[Callable[[int, int], bool]] = None) -> List[Tuple[int, int]]:
    """NVLink-connected pairs among the first ``world_size`` visible GPUs.

    ``nvml``, ``bus_ids`` and ``can_access`` replace the NVML module, the
    visible devices' PCI bus ids and the CUDA peer-access query (tests).
    """
    try:
        if bus_ids is None:
            bus_ids = _visible_pci_bus_ids()
        n = min(int(world_size), len(bus_ids))
        if n < 2:
            return []
        bus_ids = list(bus_ids)[:n]
        if nvml is None:
            try:
                import pynvml as nvml  # nvidia-ml-py
            except ImportError:
                nvml = None
        if nvml is not None:
            try:
                return sorted(_nvml_pairs(nvml, bus_ids))
            except Exception as exc:  # noqa: BLE001 - NVML missing or refusing: fall back
                logger.info("NVML NVLink query failed (%s); using CUDA peer access", exc)
        query = can_access or _kvx_can_access
        return sorted((a, b) for a in range(n) for b in range(a + 1, n) if query(a, b) and query(b, a))
    except Exception as exc:  # noqa: BLE001 - best effort, like the reference
        logger.warning("NVLink topology detection failed: %s", exc)
        return []
