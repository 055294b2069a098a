"""The B200 pair microbenchmark keeps the reference benchmark's contract
(LMPool tests/test_benchmark_kv_transfer.py: sweep parsing, JSON schema,
default Qwen geometry), so LMPool's profile builder can read its output."""
import json

import pytest

from lmpool_b200 import benchmark_kv_transfer as bk
from tests.conftest import device_count


def test_block_count_sweep_is_parsed_stably():
    assert bk.parse_block_counts("", 2) == [2]
    assert bk.parse_block_counts("1,2,4,2,1", 9) == [1, 2, 4]
    with pytest.raises(ValueError):
        bk.parse_block_counts("1,0", 2)


def test_default_geometry_matches_the_reference_defaults():
    # benchmark_kv_transfer.py:250-253 (L=28, H=8, D=128), :204-236 (block_size 256, float16 without a model)
    args = bk.parse_args([])
    assert (args.num_layers, args.num_kv_heads, args.head_dim, args.block_size) == (28, 8, 128, 256)
    assert args.resolved_dtype == "float16"


def test_metadata_has_what_the_profile_builder_reads():
    # transfer_profile.py:53-80 reads metadata.resolved_config and metadata.model.label
    meta = bk.build_metadata(bk.parse_args(["--num-layers", "36", "--dtype", "bfloat16"]))
    rc = meta["resolved_config"]
    for key in ("num_layers", "block_size", "num_kv_heads", "head_dim", "torch_dtype", "kv_dtype_bytes"):
        assert key in rc
    assert rc["num_layers"] == 36 and rc["torch_dtype"] == "bfloat16" and rc["kv_dtype_bytes"] == 2
    assert meta["model"]["label"]
    assert meta["transfer_mode"] in ("pull", "push") and meta["transfer_mode"] in meta["implementation"]
    json.dumps(meta)


@pytest.mark.gpu
@pytest.mark.skipif(device_count() < 2, reason="needs 2 GPUs")
def test_pair_sweep_runs_validates_and_writes_the_reference_schema(require_gpu, tmp_path):
    out = tmp_path / "kv_transfer.json"
    results = bk.main(["--num-layers", "4", "--block-size", "16", "--num-kv-heads", "2", "--head-dim", "64",
                       "--dtype", "bfloat16", "--block-counts", "1,3", "--iterations", "3", "--warmup", "1",
                       "--output-json", str(out)])
    assert [r["num_transfer_blocks"] for r in results] == [1, 3]
    payload = json.loads(out.read_text())
    per_block = 4 * 2 * 16 * 2 * 64 * 2
    for row in payload["results"]:
        # transfer_profile.py:63-69, :83-108: consistent bytes per block, positive latencies
        assert row["bytes_per_iteration"] == row["num_transfer_blocks"] * per_block
        assert row["mean_latency_ms"] > 0 and row["p95_latency_ms"] > 0 and row["p50_latency_ms"] > 0
        assert row["data_validation"] == "passed"
        assert row["device_mean_latency_ms"] > 0
