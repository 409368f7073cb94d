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
    """roofline.traffic comes from profiles/traffic.json under "<kernel label>/<launch shape>":
    every label the tensor-core configurations report at one GPU has its ncu figure."""
    c4, c5, x1 = (workloads.ALL_CONFIGS[n] for n in ("C4", "C5", "X1"))
    for label, cfg, rows in (("gemm_bf16_tc_pair_kernel<512>", c4, (0, 8192)), ("flash_fwd_tc_kernel", c5, (0, 128)),
                             ("conv2d_tc_kernel", x1, (0, 32))):
        traffic = bench.load_traffic(label, bench.launch_shape(cfg, rows))
        assert isinstance(traffic, int) and traffic > 0, (label, rows)
    assert bench.load_traffic("no_such_kernel", bench.launch_shape(c4, (0, 8192))) is None


def test_a_shard_never_reports_the_full_problem_traffic():
    """At N > 1 a rank launches on its own rows: the traffic lookup keys on that launch's shape,
    so a 1024-row shard gets a 1024-row capture or nothing, never the 8192-row figure."""
    c4 = workloads.ALL_CONFIGS["C4"]
    full = bench.launch_shape(c4, (0, 8192))
    assert full == "M8192_N8192_K8192"
    kernel = "gemm_bf16_tc_pair_kernel<512>"
    full_bytes = bench.load_traffic(kernel, full)
    for world in (2, 4, 8):
        rows = bench.shard_range(8192, 0, world)
        shape = bench.launch_shape(c4, rows)
        assert shape == f"M{8192 // world}_N8192_K8192"
        for label in (kernel, "gemm_bf16_tc_pair_kernel<256>", "gemm_bf16_tc_pair_kernel<480>"):
            t = bench.load_traffic(label, shape)
            assert t is None or t < full_bytes, (label, shape, t)
    c5 = workloads.ALL_CONFIGS["C5"]
    assert bench.launch_shape(c5, bench.shard_range(128, 3, 8)) == "BH16_S8192_D128_causal"


def test_every_shard_launch_of_the_scaling_run_has_its_own_capture():
    """The N = 2 / 4 / 8 launches each have a capture of their own shape (the tile width the
    library picks: 256 columns for 4096 rows, 480 for 2048 and 1024 rows), smaller than the full
    problem's, and C5's 16-plane shard at N = 8 too."""
    c4, c5 = workloads.ALL_CONFIGS["C4"], workloads.ALL_CONFIGS["C5"]
    full = bench.load_traffic("gemm_bf16_tc_pair_kernel<512>", "M8192_N8192_K8192")
    for world, label in ((2, "gemm_bf16_tc_pair_kernel<256>"), (4, "gemm_bf16_tc_pair_kernel<480>"), (8, "gemm_bf16_tc_pair_kernel<480>")):
        t = bench.load_traffic(label, bench.launch_shape(c4, bench.shard_range(8192, 0, world)))
        assert isinstance(t, int) and 0 < t < full, (world, t)
    t5 = bench.load_traffic("flash_fwd_tc_kernel", bench.launch_shape(c5, bench.shard_range(128, 0, 8)))
    assert isinstance(t5, int) and 0 < t5 < bench.load_traffic("flash_fwd_tc_kernel", "BH128_S8192_D128_causal")


def test_replicated_configurations_count_one_replica():
    """C2 (batch 1) cannot be split: at N > 1 every rank computes the same problem, and the job's
    work is one replica's, not N times it; sharded configurations sum their shards."""
    c2, c4, x1 = (workloads.ALL_CONFIGS[n] for n in ("C2", "C4", "X1"))
    assert not bench.replicated(c2, 1)
    for world in (2, 4, 8):
        assert bench.replicated(c2, world)
        assert bench.job_flops(c2.flops, c2, world) == c2.flops  # no collective is needed for replicas
        assert not bench.replicated(c4, world) and not bench.replicated(x1, world)
    assert bench.job_flops(123.0, c4, 1) == 123.0


def test_sampled_gather_blocks_cover_every_rank():
    for total, world, block in ((8192, 8, 256), (128, 8, 2), (7, 3, 4)):
        blocks = bench.sample_blocks(total, world, block)
        assert len(blocks) == world
        for r, (r0, r1) in enumerate(blocks):
            b0, b1 = bench.shard_range(total, r, world)
            assert r0 == b0 and b0 < r1 <= b1 and r1 - r0 <= block


def test_clock_csv_goes_to_a_temporary_directory(tmp_path, monkeypatch):
    monkeypatch.setenv("KG_CLOCKS_DIR", str(tmp_path))
    sampler = bench.ClockSampler(0)
    with sampler:
        pass
    if sampler.path is not None:
        assert sampler.path.parent == tmp_path


def test_launch_count_per_step_follows_the_kernel():
    assert bench.launches_per_step("conv2d_tc_kernel") == 2  # repack + conv
    for label in ("gemm_bf16_tc_pair_kernel<512>", "gemm_bf16_tc_pair_kernel<256>", "flash_fwd_tc_kernel", "matmul_simt_kernel<f32>"):
        assert bench.launches_per_step(label) == 1
