"""bench.py's host logic, without a GPU: argument defaults, the workload description of every
configuration, and the per-rank FLOP accounting of each sharding."""

from __future__ import annotations

import bench
from kernelcode_generate_b200 import workloads


def test_defaults_keep_the_driver_contract():
    args = bench.parse_args([])
    assert args.gpus == 1 and args.impl == "ours" and args.config == "C4"
    assert args.warmup >= 3 and args.steps >= 1


def test_workload_config_describes_every_configuration():
    for n in (1, 2, 8):
        for cfg in workloads.ALL_CONFIGS.values():
            c = bench.workload_config(cfg, n)
            assert c["workload"].startswith(cfg.name)
            assert c["parallelism"] == f"shard{n}"
            assert "L2 flush" in c["l2"]
    assert bench.workload_config(workloads.ALL_CONFIGS["X1"], 8)["sharding"] == "batch"
    assert bench.workload_config(workloads.CONFIGS["C2"], 8)["sharding"] == "replicas (batch 1)"


def test_extension_workload_is_not_a_baseline_config():
    assert set(workloads.CONFIGS) == {"C1", "C2", "C3", "C4", "C5"}
    x1 = workloads.ALL_CONFIGS["X1"]
    s = x1.shape
    HO = s["XH"] + s["pads"][0] + s["pads"][1] - (s["KH"] - 1)
    WO = s["XW"] + s["pads"][2] + s["pads"][3] - (s["KW"] - 1)
    assert x1.flops == 2 * s["B"] * s["F"] * HO * WO * s["C"] * s["KH"] * s["KW"]
    assert "extension" in x1.note


def test_batch_shards_cover_the_batch_once():
    B = workloads.ALL_CONFIGS["X1"].shape["B"]
    for world in (1, 2, 4, 8):
        spans = [bench.shard_range(B, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == B
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert sum(b - a for a, b in spans) == B


def test_committed_traffic_matches_the_kernel_labels_the_bench_reports():
    """roofline.traffic comes from profiles/traffic.json under "<kernel label>/<config>": every
    label the tensor-core configurations report today has its ncu figure."""
    for label, config in (("gemm_bf16_tc_pair_kernel<512>", "C4"), ("flash_fwd_tc_kernel", "C5"), ("conv2d_tc_kernel", "X1")):
        traffic = bench.load_traffic(label, config)
        assert isinstance(traffic, int) and traffic > 0, (label, config)
    assert bench.load_traffic("no_such_kernel", "C4") is None


def test_launch_count_per_step_follows_the_kernel():
    assert bench.launches_per_step("conv2d_tc_kernel") == 2  # repack + conv
    for label in ("gemm_bf16_tc_pair_kernel<512>", "gemm_bf16_tc_pair_kernel<256>", "flash_fwd_tc_kernel", "matmul_simt_kernel<f32>"):
        assert bench.launches_per_step(label) == 1
