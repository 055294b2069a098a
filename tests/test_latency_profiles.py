"""The B200 transfer-latency profiles shipped for LMPool's admission model.

Each ``latency_profile_b200_*.json`` was built by LMPool's own, unchanged
profile builder (benchmarks/build_transfer_profile.py, which calls
transfer_profile.py:113-196) from the pair microbenchmark JSON beside it
(``kv_b200_*.json``, written by ``lmpool_b200.benchmark_kv_transfer`` on two
B200s). These checks restate what LMPool's loader and scheduler rely on
(transfer_profile.py:293-330, global_scheduler.py:1349-1535): schema and
type, a geometry whose ``bytes_per_block`` equals the runtime's
``kv_transfer_bytes(1)``, and non-decreasing piecewise-linear points.
"""
import json
from pathlib import Path

import pytest

DIR = Path(__file__).resolve().parent.parent / "lmpool_b200" / "latency_profiles"
NAMES = ["qwen3_0.6b_pull", "qwen3_0.6b_push", "qwen3_8b_pull"]
LAYERS = {"qwen3_0.6b": 28, "qwen3_8b": 36}


def _load(kind: str, name: str) -> dict:
    return json.loads((DIR / f"{kind}_{name}.json").read_text())


@pytest.mark.parametrize("name", NAMES)
def test_profile_matches_its_microbenchmark_and_the_runtime_geometry(name):
    prof = _load("latency_profile_b200", name)
    bench = _load("kv_b200", name)
    model, mode = name.rsplit("_", 1)
    L = LAYERS[model]

    # transfer_profile.py:302-309: schema and type the loader accepts
    assert prof["schema_version"] == 1
    assert prof["profile_type"] == "piecewise_linear_kv_transfer_latency"
    assert prof["latency_metric"] == "p95_latency_ms"

    # model_runner.py:808-820: n * L * (bs*H*D*itemsize) * 2
    geo = prof["kv_geometry"]
    assert (geo["num_layers"], geo["block_size"], geo["num_kv_heads"], geo["head_dim"]) == (L, 256, 8, 128)
    assert geo["dtype"] == "bfloat16" and geo["kv_dtype_bytes"] == 2
    assert geo["bytes_per_block"] == L * 256 * 8 * 128 * 2 * 2

    # the microbenchmark ran this package in the mode the file names, on B200s
    meta = bench["metadata"]
    assert meta["transfer_mode"] == mode and "lmpool_b200" in meta["implementation"]
    assert all("B200" in g for g in meta["environment"]["gpus"])
    rows = {r["num_transfer_blocks"]: r for r in bench["results"]}
    assert all(r["data_validation"] == "passed" for r in rows.values())

    # transfer_profile.py:84-110: sorted, non-decreasing, p95 of the input rows
    for points in (prof["default_points"], prof["pairs"]["0,1"]["points"]):
        blocks = [p["blocks"] for p in points]
        assert blocks == sorted(rows) == [1, 2, 4, 8, 16, 32, 64]
        lat = [p["latency_ms"] for p in points]
        assert all(b >= a for a, b in zip(lat, lat[1:]))
        for p in points:
            assert p["bytes"] == p["blocks"] * geo["bytes_per_block"]
            assert p["raw_latency_ms"] == pytest.approx(rows[p["blocks"]]["p95_latency_ms"])
            assert p["latency_ms"] >= p["raw_latency_ms"]
    assert prof["pairs"]["0,1"]["logical_pair"] == [0, 1]
