"""Benchmark of the B200 structured Look attention (and companion workloads).

Default workload (one step = one Look-attention forward over one batch):
  look_cfg4   B=64, H=6, N=1025 (CLS + 32x32 offset-row hex lattice), D=64,
              bf16, Look field 8 directions x 4 rings per (batch, head, query),
              Q/K/V ~ N(0,1)/8, field ~ U(-1,1)  -> metric: Look-attn TFLOP/s

Other workloads (--workload): look_cfg1 (B8 H3 N197 fp32, 12x4 field),
negative_l1 (M=256*196, P=576, F=1728 fp32).

Contract: ``python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]``;
for N>1 launch one process per GPU with torchrun.  Each rank runs the full
per-GPU workload (weak scaling, no collective on the data path); rank 0
prints one JSON line.  Timing: CUDA events on the launching stream around
every step, L2 flushed (256 MiB write) between steps outside the events,
barrier + synchronize on both sides of the timed loop, max over ranks.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# DRAM bytes (read + write) of one sla_tc_kernel launch at look_cfg4, from the
# ncu capture summarised in profiles/look_attention_cfg4_tc.md (None = not captured).
CFG4_TRAFFIC_BYTES = None


def _peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data["hbm_gbs"], "bf16_tflops": data["bf16_tflops"],
                "bf16_tflops_sustained": data.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock / throttle sampling while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.proc is None or self.path is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        sm = [float(r[1]) for r in rows]
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


# --------------------------------------------------------------------------- workloads
class LookWorkload:
    """One Look-attention forward over a batch of synthetic inputs."""

    def __init__(self, name: str, device: torch.device, seed: int):
        from intp_preliminary_b200 import LookSlots, hexgrid

        if name == "look_cfg4":
            self.batch, self.heads, rows, cols, self.n_dir, self.dtype = 64, 6, 32, 32, 8, torch.bfloat16
        elif name == "look_cfg1":
            self.batch, self.heads, rows, cols, self.n_dir, self.dtype = 8, 3, 14, 14, 12, torch.float32
        else:
            raise ValueError(name)
        self.name, self.rows, self.cols, self.n_rad, self.dim = name, rows, cols, 4, 64
        self.patches = rows * cols
        self.seq = self.patches + 1
        self.n_slots = self.n_dir * self.n_rad
        self.scale = 1.0 / math.sqrt(self.dim)
        self.slots_table = hexgrid.synthetic_look_slots(rows, cols, self.n_dir, self.n_rad)
        self.slots = LookSlots(self.slots_table, self.n_slots)
        g = torch.Generator(device=device).manual_seed(seed)
        shape = (self.batch, self.heads, self.seq, self.dim)
        self.q, self.k, self.v = ((torch.randn(shape, device=device, generator=g) / 8).to(self.dtype) for _ in range(3))
        self.pose = torch.rand(self.batch, self.patches, self.heads, self.n_slots, device=device, generator=g) * 2 - 1
        self.out = torch.empty(shape, dtype=self.dtype, device=device)
        self.device = device
        self.slots.device_packed(device)

    @property
    def flops(self) -> float:
        return 4.0 * self.batch * self.heads * self.seq * self.seq * self.dim

    @property
    def config(self) -> dict:
        return {"workload": f"{self.name}: Look attention B{self.batch} H{self.heads} N{self.seq} D{self.dim} "
                            f"{str(self.dtype).split('.')[-1]}, {self.n_dir}x{self.n_rad} Look field "
                            f"({self.rows}x{self.cols} hex lattice + CLS)",
                "batch": self.batch, "heads": self.heads, "seq": self.seq, "head_dim": self.dim,
                "look_slots": self.n_slots}

    def step(self):
        from intp_preliminary_b200 import look_attention_forward

        look_attention_forward(self.q, self.k, self.v, self.pose, self.slots, scale=self.scale, out=self.out)

    def input_tensors(self):
        return [self.q, self.k, self.v, self.pose]

    def e2e_step(self, host_inputs, host_out):
        """Public API with host buffers: H2D copies, forward, D2H of the result."""
        from intp_preliminary_b200 import structured_look_attention

        q, k, v, pose = (h.to(self.device, non_blocking=True) for h in host_inputs)
        out = structured_look_attention(q, k, v, pose, self.slots, scale=self.scale)
        host_out.copy_(out, non_blocking=True)

    def cpu_reference(self, sample_batch: int = 1, sample_heads: int = 1) -> tuple[float, str]:
        """Time the oracle (the reference's CPU algorithm: one-hot fields einsum) on a sample."""
        from oracle.look_attention import onehot_fields, reference_structured_look_attention

        b, h = sample_batch, sample_heads
        q, k, v = (t[:b, :h].float().cpu().to(self.dtype) for t in (self.q, self.k, self.v))
        pose = self.pose[:b, :, :h].cpu()
        fields = torch.from_numpy(onehot_fields(self.slots_table, self.n_slots, h))
        reference_structured_look_attention(q, k, v, pose, fields, scale=self.scale)  # warm
        times = []
        t_end = time.perf_counter() + 10.0
        while time.perf_counter() < t_end or len(times) < 3:
            t0 = time.perf_counter()
            reference_structured_look_attention(q, k, v, pose, fields, scale=self.scale)
            times.append(time.perf_counter() - t0)
            if len(times) >= 50:
                break
        t = statistics.median(times)
        flops = 4.0 * b * h * self.seq * self.seq * self.dim
        return flops / t / 1e12, f"B{b} H{h} slice of {self.name}, median of {len(times)} runs"


class NegativeL1Workload:
    def __init__(self, device: torch.device, seed: int, features: int = 1728):
        g = torch.Generator(device=device).manual_seed(seed)
        self.rows, self.protos, self.features = 256 * 196, 576, features
        self.x = torch.randn(self.rows, features, device=device, generator=g)
        self.w = torch.randn(self.protos, features, device=device, generator=g) * 0.5
        self.out = torch.empty(self.rows, self.protos, device=device)
        self.device = device
        self.dtype = torch.float32

    @property
    def flops(self) -> float:  # one subtract + one |.|-add per (m, p, f)
        return 2.0 * self.rows * self.protos * self.features

    @property
    def bytes(self) -> float:
        return 4.0 * (self.rows * self.features + self.protos * self.features + self.rows * self.protos)

    @property
    def config(self) -> dict:
        return {"workload": f"negative_l1: x ({self.rows}, {self.features}) fp32 vs prototypes ({self.protos}, "
                            f"{self.features})", "rows": self.rows, "protos": self.protos, "features": self.features}

    def step(self):
        from intp_preliminary_b200 import negative_l1_forward

        negative_l1_forward(self.x, self.w, out=self.out)

    def input_tensors(self):
        return [self.x, self.w]

    def e2e_step(self, host_inputs, host_out):
        from intp_preliminary_b200 import negative_l1_distance

        x, w = (h.to(self.device, non_blocking=True) for h in host_inputs)
        host_out.copy_(negative_l1_distance(x, w), non_blocking=True)

    def cpu_reference(self) -> tuple[float, str]:
        from oracle.negative_l1 import negative_l1_torch

        rows = 2048
        x, w = self.x[:rows].cpu(), self.w.cpu()
        negative_l1_torch(x, w)
        times = []
        t_end = time.perf_counter() + 10.0
        while time.perf_counter() < t_end or len(times) < 3:
            t0 = time.perf_counter()
            negative_l1_torch(x, w)
            times.append(time.perf_counter() - t0)
        t = statistics.median(times)
        return 2.0 * rows * self.protos * self.features / t / 1e12, f"{rows} rows of negative_l1, -cdist p=1"


# --------------------------------------------------------------------------- timing
def _dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def _barrier(world: int):
    if world > 1:
        torch.distributed.barrier()


def _max_over_ranks(value: float, world: int, device) -> float:
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def _timed_steps(step, steps: int, warmup: int, world: int, device, flush: torch.Tensor) -> list[float]:
    stream = torch.cuda.current_stream(device)
    for _ in range(warmup):
        step()
    torch.cuda.synchronize(device)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    _barrier(world)
    torch.cuda.synchronize(device)
    for i in range(steps):
        flush.fill_(i & 0xFF)  # 256 MiB write: evicts inputs from the 126 MB L2
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize(device)
    _barrier(world)
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


def run_ours(args) -> None:
    rank, world, local = _dist_setup(args.gpus)
    device = torch.device("cuda", local if world > 1 else 0)
    from intp_preliminary_b200 import check_device_status

    if args.workload.startswith("look"):
        work = LookWorkload(args.workload, device, seed=1234 + rank)
    else:
        work = NegativeL1Workload(device, seed=1234 + rank)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    visible = [v for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    gpu_index = visible[local] if local < len(visible) else str(local)
    with ClockSampler(gpu_index) as clocks:
        times = _timed_steps(work.step, args.steps, args.warmup, world, device, flush)
    check_device_status(device)
    total_ms = _max_over_ranks(sum(times), world, device)
    ms_per_step = total_ms / args.steps
    peaks = _peaks()
    per_launch_ms = statistics.mean(times)
    if isinstance(work, LookWorkload):
        value = work.flops * world * args.steps / (total_ms * 1e-3) / 1e12
        unit, metric = "TFLOP/s", "Look-attn TFLOP/s (algorithmic 4*B*H*N^2*D)"
        achieved = work.flops / (per_launch_ms * 1e-3) / 1e12
        roofline = {"bound": "tensor", "achieved": round(achieved, 2), "peak": peaks["bf16_tflops"],
                    "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4),
                    "peak_source": f"{peaks['source']} bf16 dense (burst, kernel timed alone)",
                    "traffic": CFG4_TRAFFIC_BYTES if work.name == "look_cfg4" else None,
                    "kernel": "sla_tc_kernel" if work.dtype != torch.float32 else "sla_simt_kernel"}
    else:
        value = work.flops * world * args.steps / (total_ms * 1e-3) / 1e12
        unit, metric = "TFLOP/s", "negative-L1 FP32 op/s (2*M*P*F)"
        gbs = work.bytes / (per_launch_ms * 1e-3) / 1e9
        roofline = {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": round(gbs / peaks["hbm_gbs"], 4), "traffic": None, "kernel": "nl1_kernel",
                    "note": "FP32-issue bound; see fp32 fraction",
                    "fp32_tops": round(work.flops / (per_launch_ms * 1e-3) / 1e12, 2)}

    # End-to-end through the public API with pinned host buffers.
    host_inputs = [t.cpu().pin_memory() for t in work.input_tensors()]
    out_shape = work.out.shape
    host_out = torch.empty(out_shape, dtype=work.out.dtype).pin_memory()
    e2e_times = _timed_steps(lambda: work.e2e_step(host_inputs, host_out), args.steps, args.warmup, world, device,
                             flush)
    e2e_total = _max_over_ranks(sum(e2e_times), world, device)
    e2e_value = work.flops * world * args.steps / (e2e_total * 1e-3) / 1e12
    h2d = sum(t.numel() * t.element_size() for t in host_inputs)
    d2h = host_out.numel() * host_out.element_size()

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        cpu_value, sample = work.cpu_reference()
        cpu = {"value": round(cpu_value, 6), "unit": unit, "cores": torch.get_num_threads(), "kind": "port",
               "sample": sample}
    if rank == 0:
        line = {
            "metric": metric, "value": round(value, 3), "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": {torch.bfloat16: "bf16", torch.float32: "f32"}[work.dtype],
            "data": "synthetic (seeded; BASELINE shapes and distributions)",
            "config": {**work.config, "parallelism": f"independent replicas x{world} (weak)",
                       "l2": "flushed between steps (256 MiB write outside the timed events)"},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 4), "unit": unit, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": args.steps,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    device = torch.device("cpu")
    if args.workload.startswith("look"):
        work = _CpuLook(args.workload)
    else:
        raise SystemExit("reference arm implemented for the Look workloads")
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        work.step()
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(dt)
    value = work.sample_flops * len(times) / sum(times) / 1e12
    line = {
        "impl": "reference", "metric": "Look-attn TFLOP/s (algorithmic 4*B*H*N^2*D)", "value": round(value, 6),
        "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * sum(times) / len(times), 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": work.dtype_name, "data": "synthetic", "config": work.config,
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": work.sample},
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    del device


class _CpuLook:
    """The reference's CPU path (oracle port: one-hot fields einsum) on a bounded
    per-step sample of the Look workload: one (batch, head) slice per step."""

    def __init__(self, name: str):
        from intp_preliminary_b200 import hexgrid
        from oracle.look_attention import onehot_fields

        if name == "look_cfg4":
            batch, heads, rows, cols, n_dir, dtype = 64, 6, 32, 32, 8, torch.bfloat16
        else:
            batch, heads, rows, cols, n_dir, dtype = 8, 3, 14, 14, 12, torch.float32
        patches = rows * cols
        self.seq, self.dim = patches + 1, 64
        n_slots = n_dir * 4
        g = torch.Generator().manual_seed(1234)
        self.q, self.k, self.v = ((torch.randn(1, 1, self.seq, 64, generator=g) / 8).to(dtype) for _ in range(3))
        self.pose = torch.rand(1, patches, 1, n_slots, generator=g) * 2 - 1
        self.fields = torch.from_numpy(onehot_fields(hexgrid.synthetic_look_slots(rows, cols, n_dir, 4), n_slots, 1))
        self.sample_flops = 4.0 * self.seq * self.seq * self.dim
        self.dtype_name = "bf16" if dtype == torch.bfloat16 else "f32"
        self.config = {"workload": f"{name}: Look attention B{batch} H{heads} N{self.seq} D64 ({n_dir}x4 Look field)",
                       "batch": batch, "heads": heads, "seq": self.seq, "head_dim": 64}
        self.sample = f"one (batch, head) slice of {name} per step (B1 H1 N{self.seq})"

    def step(self):
        from oracle.look_attention import reference_structured_look_attention

        reference_structured_look_attention(self.q, self.k, self.v, self.pose, self.fields, scale=0.125)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--workload", choices=["look_cfg4", "look_cfg1", "negative_l1"], default="look_cfg4")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    args = parser.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
