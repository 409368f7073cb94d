"""Benchmark: TFLOP/s and fraction of B200 tensor peak for the reference's kernels.

    python bench.py [--gpus N --steps K --warmup W] [--config C4] [--impl ours|reference] [--no-suite]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N --steps K --warmup W

One step = one pass of the hot path over one batch of synthetic input. The headline workload
is C4 (matmul, bf16 in / fp32 out, 8192^3), sharded by contiguous row blocks of M across ranks
(total work fixed: strong scaling; no collective on the data path). Rank 0 prints ONE JSON line.

Timing: W untimed warm-up steps; then K steps, each bracketed by CUDA events on the launch
stream, with a 256 MiB L2 flush (torch fill) between steps outside the events; barrier +
synchronize around the timed loop; the max over ranks of the summed step time is the job time.
A configuration whose batch cannot be split (batch 1 at N > 1) runs as replicas: every rank
computes the same problem, and the job's work is one replica's.

Beside the timed loop:
* `e2e` repeats the metric through the reference-facing slot ABI with pinned HOST buffers: every
  step uploads the step's inputs, runs the kernel and downloads the result. At N > 1 matmul uses
  `sharding.matmul_rows_from_host`: each rank uploads its A rows and 1/N of B, one NCCL
  all-gather replicates B, and the slot entry runs the rank's rows; after the loop a sampled row
  block of the downloaded result is compared bit for bit with the device-path launch.
* `sustained` runs the headline kernel back to back for a few seconds with the clocks sampled, to
  show the rate the 1 kW power cap allows over a long run.
* `gather` (N > 1) all-gathers the sharded output into one tensor per rank over NCCL and checks
  sampled blocks of it bit for bit against launches of those blocks alone.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

from kernelcode_generate_b200.sharding import gather_rows, shard_range

ROOT = Path(__file__).resolve().parent
METRIC = "TFLOP/s and % of B200 tensor peak for matmul/conv2d/flash-attn at 1/2/4/8 GPU"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="C4", choices=["C1", "C2", "C3", "C4", "C5", "X1"],
                    help="C1-C5: the BASELINE configurations; X1: the bf16 tensor-core conv2d extension workload")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-suite", action="store_true", help="skip the other configurations")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end measurement")
    ap.add_argument("--no-gather", action="store_true",
                    help="at N > 1, skip the NCCL all-gather of the sharded output after the timed loop")
    ap.add_argument("--sustained-seconds", type=float, default=2.5,
                    help="length of the back-to-back run of the headline kernel (0 skips it)")
    ap.add_argument("--shard-of", type=int, default=None,
                    help="on one GPU, run rank 0's shard of a job with this many ranks (to time or profile one rank's launch)")
    return ap.parse_args(argv)


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {k: float(data[k]) for k in FALLBACK_PEAKS if k in data}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def launch_shape(cfg, rows) -> str:
    """The problem one launch of this rank solves, as the key of its DRAM-traffic figure:
    matmul M{rows}_N_K, attention BH{pairs}_S_D_{causal|full}, conv2d B{images}_C_HxW_F_KHxKW_s."""
    s = cfg.shape
    n = rows[1] - rows[0]
    if cfg.kernel == "matmul":
        return f"M{n}_N{s['N']}_K{s['K']}"
    if cfg.kernel == "flash_attention":
        return f"BH{n}_S{s['S']}_D{s['D']}_{'causal' if s['causal'] else 'full'}"
    return f"B{n}_C{s['C']}_{s['XH']}x{s['XW']}_F{s['F']}_{s['KH']}x{s['KW']}_s{s['stride'][0]}x{s['stride'][1]}"


def load_traffic(kernel: str, shape: str):
    """DRAM bytes per launch of `kernel` on the launch shape `shape` from the committed ncu
    summaries (profiles/traffic.json), or None when no capture of that kernel on that shape exists."""
    path = ROOT / "profiles" / "traffic.json"
    if not path.exists():
        return None
    entry = json.loads(path.read_text()).get(f"{kernel}/{shape}")
    return None if entry is None else entry.get("dram_bytes_per_launch")


def replicated(cfg, world: int) -> bool:
    """True when the configuration cannot be split across `world` ranks and every rank computes
    the whole problem (conv2d with fewer images than ranks, e.g. C2's batch of 1)."""
    return world > 1 and cfg.kernel == "conv2d" and cfg.shape["B"] < world


def job_flops(per_rank_flops: float, cfg, world: int) -> float:
    """Algorithmic work of the whole job: the ranks' shards summed, or one replica's work when the
    ranks replicate the problem (replicas add no work to the job)."""
    if replicated(cfg, world):
        return float(per_rank_flops)
    return reduce_sum(float(per_rank_flops), world)


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region, into a temporary file
    ($KG_CLOCKS_DIR when set)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int, period_ms: int = 20):
        self.device_index = device_index
        self.period_ms = period_ms
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            out_dir = Path(os.environ.get("KG_CLOCKS_DIR") or tempfile.mkdtemp(prefix="kg_clocks_"))
            out_dir.mkdir(parents=True, exist_ok=True)
            self.path = out_dir / f"clocks_rank{os.environ.get('RANK', '0')}_{os.getpid()}_{time.monotonic_ns()}.csv"
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms",
                                          str(self.period_ms), "-i", str(self.device_index)], stdout=self.fh, stderr=subprocess.DEVNULL)
            time.sleep(0.25)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None or self.path is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, power, mx, reasons = [], [], None, set()
        names = ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(names[1:], parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": sorted(reasons)}
        loaded = [x for x in sm if x > 0.5 * max(sm)] or sm
        return {"sm_mhz": float(np.median(loaded)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None}


# ---------------------------------------------------------------- distributed plumbing
def init_dist():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    import torch
    import torch.distributed as dist

    if world > 1:
        dist.barrier()
    if torch.cuda.is_available():
        torch.cuda.synchronize()


def _reduce(value: float, world: int, op_name: str) -> float:
    import torch
    import torch.distributed as dist

    if world == 1:
        return value
    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=getattr(dist.ReduceOp, op_name))
    return float(t.item())


def reduce_max(value: float, world: int) -> float:
    """Max over ranks (job time = the slowest rank)."""
    return _reduce(value, world, "MAX")


def reduce_sum(value: float, world: int) -> float:
    """Sum over ranks (total work of the job)."""
    return _reduce(value, world, "SUM")


def reduce_min(value: float, world: int) -> float:
    return _reduce(value, world, "MIN")


# ---------------------------------------------------------------- workloads on the device
def to_device(x, dev):
    import torch

    if x.dtype == np.uint16:
        return torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(dev)
    return torch.from_numpy(x).to(dev)


class Workload:
    """Device buffers plus a `step()` that launches the hot path once on `stream`."""

    def __init__(self, cfg, rank, world, dev):
        import torch

        from kernelcode_generate_b200 import kernels

        self.cfg = cfg
        self.kernels = kernels
        self.dev = dev
        inp = __import__("kernelcode_generate_b200.workloads", fromlist=["make_inputs"]).make_inputs(cfg)
        s = cfg.shape
        self.host = inp
        self.replicated = replicated(cfg, world)
        if cfg.kernel == "matmul":
            r0, r1 = shard_range(s["M"], rank, world)
            self.rows = (r0, r1)
            self.lhs_host = np.ascontiguousarray(inp["lhs"][r0:r1])
            self.lhs = to_device(self.lhs_host, dev)
            self.rhs = to_device(inp["rhs"], dev)
            self.out = torch.empty(r1 - r0, s["N"], device=dev)
            self.flops = 2 * (r1 - r0) * s["N"] * s["K"]
        elif cfg.kernel == "flash_attention":
            bh = s["B"] * s["H"]
            b0, b1 = shard_range(bh, rank, world)
            self.rows = (b0, b1)
            shape = (1, b1 - b0, s["S"], s["D"])
            self.q, self.k, self.v = (to_device(np.ascontiguousarray(inp[n].reshape(bh, s["S"], s["D"])[b0:b1]).reshape(shape), dev)
                                      for n in ("q", "k", "v"))
            self.out = torch.empty_like(self.q)
            self.flops = self.plane_flops(b1 - b0)
        else:  # conv2d: sharded by batch (C2 has batch 1: one replica per rank)
            b0, b1 = (0, s["B"]) if self.replicated else shard_range(s["B"], rank, world)
            self.rows = (b0, b1)
            self.x_host = np.ascontiguousarray(inp["input"][b0:b1])
            self.x = to_device(self.x_host, dev)
            self.w = to_device(inp["weight"], dev)
            self.out = torch.empty(b1 - b0, s["F"], *self.out_hw(), device=dev)
            self.flops = cfg.flops * (b1 - b0) // s["B"]
        self.shape = launch_shape(cfg, self.rows)

    def plane_flops(self, planes):
        s = self.cfg.shape
        full = 4 * s["S"] * s["S"] * s["D"] * planes
        return full // 2 if s["causal"] else full

    def out_hw(self):
        s = self.cfg.shape
        HO = (s["XH"] + s["pads"][0] + s["pads"][1] - s["dilation"][0] * (s["KH"] - 1) - 1) // s["stride"][0] + 1
        WO = (s["XW"] + s["pads"][2] + s["pads"][3] - s["dilation"][1] * (s["KW"] - 1) - 1) // s["stride"][1] + 1
        return HO, WO

    def step(self, stream):
        c, s = self.cfg, self.cfg.shape
        if c.kernel == "matmul":
            self.kernels.matmul(self.out, self.lhs, self.rhs, None, stream=stream)
        elif c.kernel == "flash_attention":
            self.kernels.flash_attention(self.out, self.q, self.k, self.v, s["scale"], s["causal"], stream=stream)
        else:
            self.kernels.conv2d(self.out, self.x, self.w, None, s["stride"], s["dilation"], s["pads"], stream=stream)

    def launch_rows(self, r0, r1):
        """A separate launch over rows [r0, r1) of the partitioned dimension (global indices),
        from the host inputs: the one-launch result that sampled blocks are compared with."""
        import torch

        c, s = self.cfg, self.cfg.shape
        if c.kernel == "matmul":
            out = torch.empty(r1 - r0, s["N"], device=self.dev)
            self.kernels.matmul(out, to_device(np.ascontiguousarray(self.host["lhs"][r0:r1]), self.dev), self.rhs, None)
        elif c.kernel == "flash_attention":
            bh = s["B"] * s["H"]
            q, k, v = (to_device(np.ascontiguousarray(self.host[n].reshape(bh, s["S"], s["D"])[r0:r1]).reshape(1, r1 - r0, s["S"], s["D"]),
                                 self.dev) for n in ("q", "k", "v"))
            out = torch.empty_like(q)
            self.kernels.flash_attention(out, q, k, v, s["scale"], s["causal"])
            out = out.reshape(r1 - r0, s["S"], s["D"])
        else:
            out = torch.empty(r1 - r0, s["F"], *self.out_hw(), device=self.dev)
            self.kernels.conv2d(out, to_device(np.ascontiguousarray(self.host["input"][r0:r1]), self.dev), self.w, None, s["stride"],
                                s["dilation"], s["pads"])
        torch.cuda.synchronize()
        return out


def time_steps(wl, steps, warmup, world, flush):
    """Returns (max-over-ranks summed step ms, this rank's per-launch mean ms, kernel name)."""
    import torch

    from kernelcode_generate_b200 import runtime

    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        wl.step(stream)
    torch.cuda.synchronize()
    kernel = runtime.last_kernel()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    barrier(world)
    for i in range(steps):
        if flush is not None:
            flush.fill_(i & 0xFF)  # evict L2 (256 MiB write), outside the timed events
        starts[i].record(stream)
        wl.step(stream)
        ends[i].record(stream)
    barrier(world)
    total = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    if runtime.device_status() != 0:
        raise RuntimeError("a kernel reported a pipeline timeout during the timed region")
    return reduce_max(total, world), total / steps, kernel


def sustained_run(wl, seconds, launch_ms, world, local, peaks):
    """The headline kernel back to back for about `seconds` (no L2 flush: A and B together exceed
    the 126 MB L2), one CUDA-event pair around the whole run, clocks sampled every 50 ms. Shows
    the rate the power cap allows over a long run, beside the per-launch burst figure."""
    import torch

    from kernelcode_generate_b200 import runtime

    launches = max(10, int(math.ceil(seconds * 1e3 / max(launch_ms, 1e-3))))
    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    with ClockSampler(local, period_ms=50) as clocks:
        start.record(stream)
        for _ in range(launches):
            wl.step(stream)
        end.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    if runtime.device_status() != 0:
        raise RuntimeError("a kernel reported a pipeline timeout during the sustained run")
    ms = reduce_max(start.elapsed_time(end), world)
    value = job_flops(wl.flops, wl.cfg, world) * launches / (ms * 1e-3) / 1e12
    clk = clocks.summary()
    per_launch = ms / launches
    out = {"seconds": round(ms / 1e3, 3), "launches": launches, "value": round(value, 2), "unit": "TFLOP/s",
           "ms_per_launch": round(per_launch, 4), "sm_mhz_median": clk.get("sm_mhz"), "reasons": clk.get("reasons"),
           "power_w_max": clk.get("power_w_max"), "clock_samples": clk.get("samples"),
           "frac_of_sustained_peak": round(value / (peaks["bf16_tflops_sustained"] * world), 4),
           "peak": peaks["bf16_tflops_sustained"], "l2": "no flush (A and B exceed L2)"}
    if clk.get("sm_mhz"):
        out["ms_x_mhz"] = round(per_launch * clk["sm_mhz"], 2)  # thousands of SM cycles per launch
    return out


def sample_blocks(total, world, block):
    """Row ranges [r0, r0 + block) at the start of every rank's shard (clipped to the shard)."""
    out = []
    for r in range(world):
        b0, b1 = shard_range(total, r, world)
        if b1 > b0:
            out.append((b0, min(b1, b0 + block)))
    return out


def gather_run(cfg, wl, world, rank):
    """All-gathers the rank's output block into the full output tensor on every rank (the
    single-tensor result north_star allows NCCL for), times it (max over ranks), and checks
    sampled blocks of every rank's part bit for bit against launches of those blocks alone."""
    import torch

    s = cfg.shape
    if cfg.kernel == "matmul":
        local, total, block = wl.out, s["M"], 256
    elif cfg.kernel == "flash_attention":
        local, total, block = wl.out.reshape(-1, s["S"], s["D"]), s["B"] * s["H"], 2
    elif not wl.replicated:
        local, total, block = wl.out, s["B"], 1
    else:
        return None  # replicas: every rank already holds the whole result
    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gather_rows(local, total)  # warm-up: the first NCCL all-gather also sets up its channels
    barrier(world)
    start.record(stream)
    full = gather_rows(local, total)
    end.record(stream)
    barrier(world)
    ms = reduce_max(start.elapsed_time(end), world)
    checked, equal = [], True
    if rank == 0:
        for r0, r1 in sample_blocks(total, world, block):
            ref = wl.launch_rows(r0, r1)
            same = bool(torch.equal(full[r0:r1], ref))
            checked.append([r0, r1])
            equal = equal and same
    equal = reduce_min(1.0 if equal else 0.0, world) == 1.0
    nbytes = int(full.numel() * full.element_size())
    return {"ms": round(ms, 4), "bytes": nbytes, "gb_per_s": round(nbytes / (ms * 1e-3) / 1e9, 1),
            "collective": "all_gather_into_tensor (NCCL over NVLink)", "shape": list(full.shape),
            "check": {"bitwise_equal": equal, "sampled_rows": checked, "against": "one launch of each sampled block on rank 0"}}


def _pinned(x):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).view(torch.bfloat16) if x.dtype == np.uint16 else torch.from_numpy(
        np.ascontiguousarray(x))
    return t.pin_memory()


def e2e_run(cfg, wl, steps, world):
    """The metric through the reference-facing slot ABI (kg_sm100_*_entry via the execute engine)
    with pinned HOST buffers: every step copies the rank's inputs H2D, runs the kernel and copies
    the result D2H inside the (synchronous) call. At N > 1 matmul goes through
    sharding.matmul_rows_from_host, which uploads only this rank's 1/N of B and replicates it over
    NVLink. Wall clock, max over ranks; bytes are per rank."""
    import torch

    from kernelcode_generate_b200 import kernels
    from kernelcode_generate_b200.sharding import matmul_rows_from_host

    s = cfg.shape
    path = f"{cfg.kernel} slot entry (kg_execute_entry ABI) on pinned host buffers, wall clock, max over ranks"
    if cfg.kernel == "matmul":
        lhs = _pinned(wl.lhs_host)
        out = torch.empty(tuple(wl.out.shape), dtype=torch.float32).pin_memory()
        if world > 1:
            k0, k1 = shard_range(s["K"], int(os.environ.get("RANK", "0")), world)
            rhs = torch.empty((s["K"], s["N"]), dtype=torch.bfloat16 if cfg.dtype == "bf16" else torch.float32)
            rhs[k0:k1] = _pinned(wl.host["rhs"][k0:k1])  # only this rank's rows of B are read
            rhs = rhs.pin_memory()
            h2d = lhs.numel() * lhs.element_size() + (k1 - k0) * s["N"] * rhs.element_size()
            call = lambda: matmul_rows_from_host(out, lhs, rhs, None, *cfg.tiles)  # noqa: E731
            path = ("matmul: each rank uploads its A rows and 1/N of B's rows, one NCCL all-gather replicates B over NVLink, "
                    "then the slot entry (kg_execute_entry ABI) runs the rank's rows from host memory; wall clock, max over ranks")
        else:
            rhs = _pinned(wl.host["rhs"])
            h2d = lhs.numel() * lhs.element_size() + rhs.numel() * rhs.element_size()
            call = lambda: kernels.matmul_inputs_dynamic_tile_dynamic_kernel(out, lhs, rhs, None, *cfg.tiles)  # noqa: E731
    elif cfg.kernel == "flash_attention":
        bh = s["B"] * s["H"]
        b0, b1 = wl.rows
        shape = (1, b1 - b0, s["S"], s["D"])
        args = [_pinned(np.ascontiguousarray(wl.host[n].reshape(bh, s["S"], s["D"])[b0:b1]).reshape(shape)) for n in ("q", "k", "v")]
        out = torch.empty(shape, dtype=args[0].dtype).pin_memory()
        h2d = sum(a.numel() * a.element_size() for a in args)
        call = lambda: kernels.flash_attention_inputs_dynamic_tile_dynamic_kernel(out, *args, *cfg.tiles, s["scale"], s["causal"])  # noqa: E731
    else:
        args = [_pinned(wl.x_host), _pinned(wl.host["weight"])]
        out = torch.empty(tuple(wl.out.shape), dtype=torch.float32).pin_memory()
        h2d = sum(a.numel() * a.element_size() for a in args)
        call = lambda: kernels.conv2d_inputs_dynamic_tile_dynamic_kernel(  # noqa: E731
            out, args[0], args[1], None, *s["stride"], *s["dilation"], *s["pads"], *cfg.tiles)
    call()  # warm-up (sizes the staging arena, sets up the NCCL channels)
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(steps):
        call()
    barrier(world)
    elapsed = reduce_max(time.perf_counter() - t0, world)
    total_flops = job_flops(float(wl.flops), cfg, world)
    d2h = out.numel() * out.element_size()
    # The downloaded result against the device-path launches of the timed loop, bit for bit.
    dev_out = wl.out.detach().cpu()
    rows = min(256, dev_out.shape[0])
    equal = bool(torch.equal(out.reshape(dev_out.shape)[:rows], dev_out[:rows]))
    equal = reduce_min(1.0 if equal else 0.0, world) == 1.0
    return {"value": round(total_flops * steps / elapsed / 1e12, 3), "unit": "TFLOP/s", "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "ms_per_step": round(elapsed / steps * 1e3, 3), "path": path,
            "check": {"bitwise_equal_to_device_path": equal, "rows_compared_per_rank": rows}}


# ---------------------------------------------------------------- CPU reference / baseline
def cpu_sample(cfg, threads, opt="O2"):
    """Runs the reference's CPU path (oracle/_ref at `opt`) or the C port on a bounded sample of
    the workload. Returns (TFLOP/s, seconds, kind, sample description, threads used).
    -O0 (how the reference's execute engine compiles: no -O flag) is about 20x slower than -O2,
    so its samples are smaller: 8-row instead of 80-row matmul bands, 16- instead of 128-row
    query tiles."""
    sys.path.insert(0, str(ROOT))
    import oracle

    kind = "reference" if oracle.ref_available(opt) else "port"
    impl = "ref" if kind == "reference" else "port"
    small = opt == "O0" and kind == "reference"
    inp = __import__("kernelcode_generate_b200.workloads", fromlist=["make_inputs"]).make_inputs(cfg)
    s = cfg.shape
    t_threads = threads if kind == "reference" else 1
    if cfg.kernel == "matmul":
        tile_h = (8 if small else 80) if cfg.dtype == "bf16" else cfg.tiles[0]
        tiles = (tile_h, 96, 72) if cfg.dtype == "bf16" else cfg.tiles
        rows = min(s["M"], tile_h * t_threads)
        t0 = time.perf_counter()
        oracle.matmul(inp["lhs"], inp["rhs"], None, tiles=tiles, rows=(0, rows), impl=impl, threads=t_threads, opt=opt)
        dt = time.perf_counter() - t0
        flops = 2 * rows * s["N"] * s["K"]
        desc = f"rows 0..{rows} of M={s['M']} (tiles {tiles}), {flops / 1e9:.1f} GFLOP"
    elif cfg.kernel == "flash_attention":
        S = s["S"]
        if S > 1024:
            br = 16 if small else 128
            tiles = (br, cfg.tiles[1])
            q_rows = (S - br * max(1, t_threads), S)  # last query tiles: the most work per row
            bh = (0, 1)
            t0 = time.perf_counter()
            oracle.flash_attention(inp["q"], inp["k"], inp["v"], tiles=tiles, scale=s["scale"], causal=s["causal"], bh=bh,
                                   q_rows=q_rows, impl=impl, threads=t_threads, opt=opt)
            dt = time.perf_counter() - t0
            n = q_rows[1] - q_rows[0]
            keys = sum((r + 1) if s["causal"] else S for r in range(q_rows[0], q_rows[1]))
            flops = 4 * keys * s["D"]
            desc = f"(b,h)=0, query rows {q_rows[0]}..{q_rows[1]} ({n} rows, tiles {tiles}), {flops / 1e9:.1f} GFLOP"
        else:
            t0 = time.perf_counter()
            oracle.flash_attention(inp["q"], inp["k"], inp["v"], tiles=cfg.tiles, scale=s["scale"], causal=s["causal"], impl=impl,
                                   threads=t_threads, opt=opt)
            dt = time.perf_counter() - t0
            flops = cfg.flops
            desc = "full workload"
    else:
        nb = 1 if s["B"] > 1 else s["B"]  # batched conv: the first image
        t0 = time.perf_counter()
        oracle.conv2d(np.ascontiguousarray(inp["input"][:nb]), inp["weight"], None, stride=s["stride"], dilation=s["dilation"],
                      pads=s["pads"], tiles=cfg.tiles, impl=impl, threads=t_threads, opt=opt)
        dt = time.perf_counter() - t0
        flops = cfg.flops * nb // s["B"]
        desc = "full workload" if nb == s["B"] else f"image 0 of {s['B']}, {flops / 1e9:.1f} GFLOP"
    return flops / dt / 1e12, dt, kind, desc, t_threads


def cpu_baseline(cfg, threads):
    """The reference's CPU path timed on this host: npu_demo helpers built -O2 (the stronger
    baseline, the headline `value`), and beside it built as the reference's execute engine builds
    them (kernel_gen/execute_engine/compiler.py:137: -std=c++17, no -O flag, i.e. -O0)."""
    v, dt, kind, desc, used = cpu_sample(cfg, threads, "O2")
    out = {"value": round(v, 6), "unit": "TFLOP/s", "cores": used, "kind": kind,
           "sample": f"{desc}; {dt:.1f} s" + ("; npu_demo helpers g++ -O2" if kind == "reference" else "; C port, 1 thread")}
    if kind == "reference":
        v0, dt0, kind0, desc0, used0 = cpu_sample(cfg, threads, "O0")
        out["as_shipped_O0"] = {"value": round(v0, 7), "unit": "TFLOP/s", "cores": used0, "kind": kind0,
                                "sample": f"{desc0}; {dt0:.1f} s; npu_demo helpers g++ -std=c++17 without -O (-O0)",
                                "o2_over_o0": round(v / v0, 2) if v0 > 0 else None}
    return out


def reference_arm(args):
    """`--impl reference`: the reference's own CPU implementation of the path on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from kernelcode_generate_b200 import workloads

    cfg = workloads.ALL_CONFIGS[args.config]
    threads = os.cpu_count() or 1
    for _ in range(args.warmup if cfg.kernel != "matmul" or cfg.dtype != "bf16" else 0):
        cpu_sample(cfg, threads)
    vals, secs = [], 0.0
    kind = desc = None
    used = threads
    for _ in range(max(1, min(args.steps, 3))):
        v, dt, kind, desc, used = cpu_sample(cfg, threads)
        vals.append(v)
        secs += dt
    value = float(np.median(vals))
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": len(vals), "warmup": args.warmup, "ms_per_step": round(secs / len(vals) * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32" if cfg.dtype == "f32" else "f32 (bf16-rounded inputs)",
        "data": "synthetic", "config": workload_config(cfg, args.gpus),
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": used, "kind": kind,
                         "sample": desc + " per step; npu_demo helpers g++ -O2" if kind == "reference" else desc},
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


NOMINAL_TF32_TFLOPS = 1100.0  # B200 dense TF32 tensor peak, nominal (no measured figure on this pool)


def fp32_peak_fractions(value_tflops: float, world: int, dev, replicas: bool = False) -> dict:
    """The fp32 configurations against the dense TF32 tensor peak and the FP32 CUDA-core peak
    (2 FLOP x 128 lanes x SMs x max SM clock), both nominal; the kernels run exact FP32 FMAs on
    CUDA cores because TF32 cannot meet rtol 1e-4 / atol 1e-5. Replicas are measured against one
    GPU's peak (the job's work is one replica's)."""
    import torch

    props = torch.cuda.get_device_properties(dev)
    try:
        clock_mhz = float(subprocess.run(["nvidia-smi", "--query-gpu=clocks.max.sm", "--format=csv,noheader,nounits", "-i",
                                          str(dev.index or 0)], capture_output=True, text=True, timeout=10).stdout.split()[0])
    except Exception:  # noqa: BLE001 - nvidia-smi missing or unparsable: the B200 nominal max clock
        clock_mhz = 1965.0
    simt = 2 * 128 * props.multi_processor_count * clock_mhz * 1e6 / 1e12
    gpus = 1 if replicas else world
    return {"frac_of_tf32_peak_nominal": round(value_tflops / (NOMINAL_TF32_TFLOPS * gpus), 6),
            "fp32_simt_peak_tflops_nominal": round(simt, 1), "frac_of_fp32_simt_peak": round(value_tflops / (simt * gpus), 4)}


def launches_per_step(kernel: str) -> int:
    """Kernels of this library one step launches: the tensor-core conv2d runs one repack kernel
    (input and weights) before the GEMM kernel; every other path is one kernel."""
    return 2 if kernel == "conv2d_tc_kernel" else 1


def workload_config(cfg, n_gpus):
    if cfg.kernel == "conv2d":
        sharding = "replicas (batch 1)" if replicated(cfg, n_gpus) else "batch"
    else:
        sharding = {"matmul": "contiguous row blocks of M", "flash_attention": "batch x heads"}[cfg.kernel]
    return {"workload": f"{cfg.name}: {cfg.note}", **{k: v for k, v in cfg.shape.items()}, "sharding": sharding,
            "parallelism": f"shard{n_gpus}", "l2": "256 MiB L2 flush between timed steps (outside the events)"}


# ---------------------------------------------------------------- main
def main(argv=None):
    args = parse_args(argv)
    if args.impl == "reference":
        return reference_arm(args)
    import torch

    from kernelcode_generate_b200 import workloads

    rank, world, local = init_dist()
    dev = torch.device("cuda", local)
    peaks, peak_src = load_peaks()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    cfg = workloads.ALL_CONFIGS[args.config]
    if args.shard_of is not None and (world != 1 or args.shard_of < 1):
        raise SystemExit("--shard-of runs one rank's shard on one GPU: use it without torchrun, with a positive rank count")
    wl = Workload(cfg, 0, args.shard_of, dev) if args.shard_of else Workload(cfg, rank, world, dev)
    with ClockSampler(local) as clocks:
        job_ms, launch_ms, kernel = time_steps(wl, args.steps, args.warmup, world, flush)
    total_flops = job_flops(float(wl.flops), cfg, world)
    value = total_flops * args.steps / (job_ms * 1e-3) / 1e12
    launch_ms_max = reduce_max(launch_ms, world)
    achieved = wl.flops / (launch_ms * 1e-3) / 1e12  # this rank's kernel, algorithmic FLOPs per launch
    tensor_peak = peaks["bf16_tflops"]
    traffic = load_traffic(kernel, wl.shape)
    sustained = None
    if args.sustained_seconds > 0 and cfg.dtype == "bf16":
        sustained = sustained_run(wl, args.sustained_seconds, launch_ms, world, local, peaks)
    gather = gather_run(cfg, wl, world, rank) if world > 1 and not args.no_gather else None
    e2e = None
    if not args.no_e2e:
        e2e = e2e_run(cfg, wl, args.e2e_steps, world)

    suite = {}
    if not args.no_suite:
        for name in ("C1", "C2", "C3", "C5", "X1"):
            if name == cfg.name:
                continue
            c = workloads.ALL_CONFIGS[name]
            w2 = Workload(c, rank, world, dev)
            steps = max(3, min(args.steps, 10))
            ms, per_launch, k2 = time_steps(w2, steps, max(3, args.warmup), world, flush)
            tot = job_flops(float(w2.flops), c, world)
            v2 = tot * steps / (ms * 1e-3) / 1e12
            gpus = 1 if w2.replicated else world
            suite[name] = {"value": round(v2, 3), "unit": "TFLOP/s", "ms_per_step": round(ms / steps, 4), "kernel": k2,
                           "launches_per_step": launches_per_step(k2), "launch_shape": w2.shape,
                           "sharding": "replicas: job work = one replica's" if w2.replicated else "sharded",
                           "frac_of_bf16_peak": round(v2 / (tensor_peak * gpus), 4), "workload": c.note}
            if c.dtype == "f32":
                suite[name].update(fp32_peak_fractions(v2, world, dev, w2.replicated))
            else:
                tr = load_traffic(k2, w2.shape)
                if tr is not None:
                    suite[name]["traffic"] = tr
            del w2
            torch.cuda.empty_cache()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(cfg, os.cpu_count() or 1)

    if rank == 0:
        gpus = 1 if wl.replicated else world
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(job_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": cfg.dtype, "data": "synthetic",
            "config": {**workload_config(cfg, world), **({"shard_of": args.shard_of} if args.shard_of else {})},
            "frac_of_peak": round(value / (tensor_peak * gpus), 4),
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": tensor_peak, "unit": "TFLOP/s",
                         "frac": round(achieved / tensor_peak, 4), "traffic": traffic, "kernel": kernel,
                         "launch_shape": wl.shape,
                         "traffic_source": "profiles/traffic.json entry for this kernel and launch shape" if traffic is not None
                         else "no ncu capture of this kernel on this launch shape",
                         "peak_source": f"{peak_src} bf16_tflops (burst)",
                         "launch_ms": round(launch_ms, 4), "launch_ms_max_over_ranks": round(launch_ms_max, 4),
                         "algorithmic_flop_per_launch": int(wl.flops)},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": args.steps * launches_per_step(kernel),
            "clocks": clocks.summary(),
            "sustained": sustained,
            "suite": suite,
        }
        if gather is not None:
            line["gather"] = gather
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
