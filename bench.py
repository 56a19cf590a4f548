"""Benchmark of the B200 SHARE-ViT Look-attention path.

Default workload (``--workload model``): one step is
the full half6d3r SHARE-ViT DeiT-Tiny inference forward over 256 images per GPU
(bf16, random-init weights, images ~ N(0, 1) 224x224x3), plus the gather of
the logits to rank 0 when N > 1 (weak scaling: 256 images per GPU).  Metric:
images/s over all GPUs.  The line also carries the Look-attention kernel timed
in place inside that forward (``roofline``) and the long-sequence Look layer (B64 H6
N1025 D64 bf16) timed on its own (``look_attention_cfg4``).

``--global-batch G`` fixes the total batch instead (strong scaling: G / N images
per GPU), the sweep of global batches 256 / 1024 / 4096 over 1 / 2 / 4 / 8 GPUs.

Other workloads: ``look_cfg4`` / ``look_cfg1`` (one Look-attention forward per
step, TFLOP/s), ``negative_l1`` (M=256*196, P=576, F=1728 fp32; ``--features``
picks 432 or the real 1344 / 336), ``dense_look_grid`` (dense Look-grid
sampling, B256 H3 on the 14x14 lattice, fp32 grids -> the (B, H, 196, 196)
bias, GB/s; its backward timed alongside) and ``reference_model`` (the
reference's own ``DeiTTinyRotHexLook`` half6d3r, unchanged, imported from
baseline/_ref with this package's operators installed under the reference's
module names, bf16 autocast, 256 images per GPU).

Contract: ``python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]``;
for N > 1 launch one process per GPU with torchrun.  Timing: CUDA events on the
launching stream around every step, L2 flushed (256 MiB write) between steps
outside the events, barrier + synchronize on both sides of the timed loop, max
over ranks; rank 0 prints one JSON line.  ``--impl reference`` times the
reference's CPU implementation on bounded samples, rank 0 only: the
reference's own model code from baseline/_ref when it is installed
(``kind: reference``), else the oracle port of its algorithm (``kind: port``).
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

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# DRAM bytes (read + write) of one sla_tc_kernel launch at look_cfg4, from one
# ncu capture of that launch (dram__bytes_read.sum + dram__bytes_write.sum).
CFG4_TRAFFIC_BYTES = int((202.150400 + 34.622976) * 1e6)
# DRAM bytes (read + write) of one sla_short_kernel launch on the model forward's
# inputs (B256 H3 N196, SLOT_FIELDS), from one ncu capture of that launch.
MODEL_ATTN_TRAFFIC_BYTES = int((70.775808 + 3.503360) * 1e6)
# DRAM bytes (read + write) of one nl1_vec_kernel launch (50176 x 576 x F), from
# one ncu capture per feature size.
NL1_TRAFFIC_BYTES = {1728: int((350.991872 + 97.320448) * 1e6), 432: int((87.734528 + 71.396864) * 1e6)}
# Algorithmic FLOPs of one half6d3r image: trunk linears (qkv, proj, fc1, fc2 over
# 196 tokens, 12 blocks), Look attention QK and PV (4 x 3 heads x 196^2 x 64 per
# block) and the tokenizer + Look-bank GEMM (195 patches x 1680 x 792).
MODEL_FLOPS_PER_IMAGE = (196 * 12 * 2 * (192 * 576 + 192 * 192 + 2 * 192 * 768)
                         + 12 * 4 * 3 * 196 * 196 * 64 + 2 * 195 * (1344 + 336) * 792)


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

    def __init__(self, gpu_index: str):
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
        power = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(power) if power else None}


# --------------------------------------------------------------------------- workloads
class ModelWorkload:
    """Full half6d3r forward over a per-GPU batch; logits gathered to rank 0."""

    name = "model"
    dtype = torch.bfloat16
    unit = "images/s"
    metric = "half6d3r SHARE-ViT DeiT-Tiny inference images/s (bf16)"

    def __init__(self, ctx, per_gpu_batch: int, seed: int):
        from intp_preliminary_b200.share_vit import ShareViTHalf6d3r

        self.ctx = ctx
        self.device = ctx.device
        self.batch = per_gpu_batch
        self.global_batch = per_gpu_batch * ctx.world
        self.model = ShareViTHalf6d3r(precision="bf16").init_weights(seed=0, look_grid_std=0.02).to(self.device)
        g = torch.Generator(device=self.device).manual_seed(seed + ctx.rank)
        self.images = torch.randn(self.batch, 3, 224, 224, device=self.device, generator=g)
        self.logits = None
        self.model(self.images[:2])  # build the rendered-prototype cache and the packed slot table
        from intp_preliminary_b200.serving import GraphedForward

        self.graphed = GraphedForward(self.model, self.images)  # the whole forward as one CUDA graph

    @property
    def units_per_step(self) -> float:
        return float(self.global_batch)

    @property
    def config(self) -> dict:
        return {"workload": f"model: half6d3r SHARE-ViT DeiT-Tiny forward, {self.batch} images of 224x224x3 per GPU, "
                            "bf16, 12 blocks x 3 heads, head_dim 64, 12x4 Look field per layer/head",
                "batch_per_gpu": self.batch, "global_batch": self.global_batch, "tokens": 196,
                "look_slots": self.model.look_slots.n_slots}

    def step(self):
        from intp_preliminary_b200.sharding import gather_to_main

        local = self.graphed.replay()
        self.logits = gather_to_main(local, self.ctx, self.global_batch)

    def eager_step(self):
        """The same forward launched kernel by kernel (for in-model kernel timing)."""
        self.model(self.images)

    def e2e_inputs(self):
        g = torch.Generator().manual_seed(4321 + self.ctx.rank)
        return [torch.randn(self.batch, 3, 224, 224, generator=g).pin_memory() for _ in range(2)]

    def e2e_output(self):
        return torch.empty(self.global_batch if self.ctx.is_main else 1, 100, dtype=torch.float32).pin_memory()

    def e2e_run(self, host_inputs, host_out, steps: int) -> float:
        """`steps` batches from pinned host memory through PipelinedInference
        (H2D of batch i+1 overlapped with the forward of batch i, logits
        gathered to rank 0 and copied back every step); device ms in total."""
        from intp_preliminary_b200.serving import PipelinedInference
        from intp_preliminary_b200.sharding import gather_to_main

        if not hasattr(self, "pipeline"):
            self.pipeline = PipelinedInference(self.model, self.batch, self.device)
        outs = [host_out] * steps
        batches = [host_inputs[i % len(host_inputs)] for i in range(steps)]
        gather = lambda i, logits: gather_to_main(logits, self.ctx, self.global_batch)  # noqa: E731
        stream = torch.cuda.current_stream(self.device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        self.pipeline.run(batches, outs, after_forward=gather)
        end.record(stream)
        torch.cuda.synchronize(self.device)
        return start.elapsed_time(end)

    def cpu_reference(self):
        return _reference_cpu_sample(2)


REFERENCE_DIR = ROOT / "baseline" / "_ref"
HALF6D3R = dict(use_pos_embed=True, directions=6, global_directions=12, angular_bins_per_radius=3,
                look_compact_variable_rings=True, tokenizer_null_initial_score=0.0)


def _reference_model_class(drop_in: bool):
    """The reference's ``DeiTTinyRotHexLook`` from baseline/_ref, with this
    package's operators under the reference's module names when ``drop_in``."""
    if not (REFERENCE_DIR / "model" / "deit_tiny_rot_hex_look.py").exists():
        return None
    if str(REFERENCE_DIR) not in sys.path:
        sys.path.insert(1, str(REFERENCE_DIR))
    if drop_in:
        from intp_preliminary_b200.layers.drop_in import install_drop_in

        install_drop_in(polar_render="torch")
    from model.deit_tiny_rot_hex_look import DeiTTinyRotHexLook

    return DeiTTinyRotHexLook


def _reference_half6d3r(drop_in: bool, look_grid_std: float = 0.02):
    """The reference model with the seeded init of ``ShareViTHalf6d3r.init_weights``."""
    from intp_preliminary_b200.share_vit import ShareViTHalf6d3r

    cls = _reference_model_class(drop_in)
    if cls is None:
        return None
    weights = ShareViTHalf6d3r(precision="fp32").init_weights(seed=0, look_grid_std=look_grid_std)
    model = cls(**HALF6D3R).eval()
    model.load_state_dict(weights.state_dict(), strict=True)
    return model


class ReferenceModelWorkload(ModelWorkload):
    """The reference's own half6d3r model, unchanged, on this package's operators
    (bf16 autocast, eager PyTorch around them); logits gathered to rank 0."""

    name = "reference_model"
    metric = "half6d3r SHARE-ViT DeiT-Tiny inference images/s (reference model code, bf16 autocast)"

    def __init__(self, ctx, per_gpu_batch: int, seed: int):
        self.ctx = ctx
        self.device = ctx.device
        self.batch = per_gpu_batch
        self.global_batch = per_gpu_batch * ctx.world
        model = _reference_half6d3r(drop_in=True)
        if model is None:
            raise SystemExit("reference_model needs the reference in baseline/_ref "
                             "(sh baseline/install_reference.sh <checkout>)")
        self.model = model.to(self.device)
        g = torch.Generator(device=self.device).manual_seed(seed + ctx.rank)
        self.images = torch.randn(self.batch, 3, 224, 224, device=self.device, generator=g)
        self.logits = None

    @property
    def config(self) -> dict:
        return {"workload": f"reference_model: the reference's DeiTTinyRotHexLook half6d3r (unchanged model code) "
                            f"on this package's operators, {self.batch} images of 224x224x3 per GPU, bf16 autocast",
                "batch_per_gpu": self.batch, "global_batch": self.global_batch, "tokens": 196}

    def forward(self, images):
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            return self.model(images)

    def step(self):
        from intp_preliminary_b200.sharding import gather_to_main

        self.logits = gather_to_main(self.forward(self.images).float(), self.ctx, self.global_batch)

    def e2e_step(self, host_inputs, host_out):
        from intp_preliminary_b200.sharding import gather_to_main

        images = host_inputs[0].to(self.device, non_blocking=True)
        logits = gather_to_main(self.forward(images).float(), self.ctx, self.global_batch)
        if self.ctx.is_main:
            host_out.copy_(logits, non_blocking=True)

    def e2e_inputs(self):
        return super().e2e_inputs()[:1]

    def cpu_reference(self):
        return _reference_cpu_sample(2)


def _reference_cpu_sample(count: int, seconds: float = 15.0):
    """images/s of the reference's own model on the host CPU (all threads),
    ``count`` images per run; falls back to the oracle port when the reference
    is not installed.  Returns (value, sample, kind)."""
    images = torch.randn(count, 3, 224, 224, generator=torch.Generator().manual_seed(1234))
    model = _reference_half6d3r(drop_in=False)
    if model is not None:
        run = lambda: model(images)  # noqa: E731
        what, kind = f"the reference's own DeiTTinyRotHexLook (baseline/_ref) on CPU, {count} images", "reference"
    else:
        from intp_preliminary_b200.share_vit import ShareViTHalf6d3r
        from oracle.share_vit_cpu import reference_forward_cpu

        port = ShareViTHalf6d3r(precision="fp32").init_weights(seed=0, look_grid_std=0.02)
        run = lambda: reference_forward_cpu(port, images)  # noqa: E731
        what, kind = f"reference CPU algorithm (oracle port: dense fields + explicit attention), {count} images", \
            "port"
    with torch.no_grad():
        run()
        times, t_end = [], time.perf_counter() + seconds
        while time.perf_counter() < t_end or len(times) < 2:
            t0 = time.perf_counter()
            run()
            times.append(time.perf_counter() - t0)
            if len(times) >= 20:
                break
    return count / statistics.median(times), f"{what}, median of {len(times)}", kind


class LookWorkload:
    """One Look-attention forward over a batch of synthetic inputs."""

    unit = "TFLOP/s"
    metric = "Look-attn TFLOP/s (algorithmic 4*B*H*N^2*D)"

    def __init__(self, name: str, device: torch.device, seed: int, world: int = 1):
        from intp_preliminary_b200 import LookSlots, hexgrid

        if name == "look_cfg4":
            self.batch, self.heads, rows, cols, self.n_dir, self.dtype = 64, 6, 32, 32, 8, torch.bfloat16
        elif name == "look_cfg1":
            self.batch, self.heads, rows, cols, self.n_dir, self.dtype = 8, 3, 14, 14, 12, torch.float32
        else:
            raise ValueError(name)
        self.name, self.rows, self.cols, self.n_rad, self.dim, self.world = name, rows, cols, 4, 64, world
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
    def units_per_step(self) -> float:
        return self.flops * self.world / 1e12

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

    @property
    def backward_flops(self) -> float:  # S = QK^T, dP = dO V^T, dV = P^T dO, dK = dS^T Q, dQ = dS K
        return 10.0 * self.batch * self.heads * self.seq * self.seq * self.dim

    def backward_prepare(self, seed: int):
        from intp_preliminary_b200 import look_attention_forward

        self.bwd_out, self.bwd_lse = look_attention_forward(self.q, self.k, self.v, self.pose, self.slots,
                                                            scale=self.scale, want_lse=True)
        g = torch.Generator(device=self.device).manual_seed(seed)
        self.grad_out = torch.randn(self.q.shape, device=self.device, generator=g).to(self.dtype)

    def backward_step(self, kernel: str = "auto"):
        from intp_preliminary_b200 import look_attention_backward

        look_attention_backward(self.q, self.k, self.v, self.bwd_out, self.bwd_lse, self.grad_out, self.pose,
                                self.slots, scale=self.scale, kernel=kernel)

    def e2e_inputs(self):
        return [t.cpu().pin_memory() for t in (self.q, self.k, self.v, self.pose)]

    def e2e_output(self):
        return torch.empty(self.out.shape, dtype=self.out.dtype).pin_memory()

    def e2e_step(self, host_inputs, host_out):
        from intp_preliminary_b200 import structured_look_attention

        q, k, v, pose = (h.to(self.device, non_blocking=True) for h in host_inputs)
        host_out.copy_(structured_look_attention(q, k, v, pose, self.slots, scale=self.scale), non_blocking=True)

    def cpu_reference(self, sample_batch: int = 1, sample_heads: int = 1):
        from oracle.look_attention import onehot_fields, reference_structured_look_attention

        b, h = sample_batch, sample_heads
        q, k, v = (t[:b, :h].float().cpu().to(self.dtype) for t in (self.q, self.k, self.v))
        pose = self.pose[:b, :, :h].cpu()
        fields = torch.from_numpy(onehot_fields(self.slots_table, self.n_slots, h))
        reference_structured_look_attention(q, k, v, pose, fields, scale=self.scale)
        times, t_end = [], time.perf_counter() + 10.0
        while time.perf_counter() < t_end or len(times) < 3:
            t0 = time.perf_counter()
            reference_structured_look_attention(q, k, v, pose, fields, scale=self.scale)
            times.append(time.perf_counter() - t0)
            if len(times) >= 50:
                break
        flops = 4.0 * b * h * self.seq * self.seq * self.dim
        return flops / statistics.median(times) / 1e12, f"B{b} H{h} slice of {self.name}, median of {len(times)} runs"


class NegativeL1Workload:
    unit = "TFLOP/s"
    metric = "negative-L1 FP32 op/s (2*M*P*F)"
    dtype = torch.float32
    name = "negative_l1"

    def __init__(self, device: torch.device, seed: int, world: int = 1, features: int = 1728):
        g = torch.Generator(device=device).manual_seed(seed)
        self.rows, self.protos, self.features, self.world = 256 * 196, 576, features, world
        self.x = torch.randn(self.rows, features, device=device, generator=g)
        self.w = torch.randn(self.protos, features, device=device, generator=g) * 0.5
        self.out = torch.empty(self.rows, self.protos, device=device)
        self.device = device

    @property
    def flops(self) -> float:  # one subtract + one |.|-add per (m, p, f)
        return 2.0 * self.rows * self.protos * self.features

    @property
    def units_per_step(self) -> float:
        return self.flops * self.world / 1e12

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

    def backward_prepare(self, seed: int):
        g = torch.Generator(device=self.device).manual_seed(seed)
        self.grad_out = torch.randn(self.out.shape, device=self.device, generator=g)

    def backward_step(self):
        from intp_preliminary_b200 import negative_l1_backward

        negative_l1_backward(self.x, self.w, self.grad_out)

    def e2e_inputs(self):
        return [self.x.cpu().pin_memory(), self.w.cpu().pin_memory()]

    def e2e_output(self):
        return torch.empty(self.out.shape, dtype=self.out.dtype).pin_memory()

    def e2e_step(self, host_inputs, host_out):
        from intp_preliminary_b200 import negative_l1_distance

        x, w = (h.to(self.device, non_blocking=True) for h in host_inputs)
        host_out.copy_(negative_l1_distance(x, w), non_blocking=True)

    def cpu_reference(self):
        from oracle.negative_l1 import negative_l1_torch

        rows = 2048
        x, w = self.x[:rows].cpu(), self.w.cpu()
        negative_l1_torch(x, w)
        times, t_end = [], time.perf_counter() + 10.0
        while time.perf_counter() < t_end or len(times) < 3:
            t0 = time.perf_counter()
            negative_l1_torch(x, w)
            times.append(time.perf_counter() - t0)
        return 2.0 * rows * self.protos * self.features / statistics.median(times) / 1e12, \
            f"{rows} rows of negative_l1, -cdist p=1"


class DenseLookGridWorkload:
    unit = "GB/s"
    metric = "dense Look-grid sampling bias throughput (algorithmic bytes / s)"
    dtype = torch.float32
    name = "dense_look_grid"

    def __init__(self, device: torch.device, seed: int, world: int = 1):
        from intp_preliminary_b200 import hexgrid, look_sampling_tables

        coords = torch.from_numpy(hexgrid.offset_row_lattice(14, 14)).float()
        self.tables = [t.to(device) for t in look_sampling_tables(coords).values()]
        self.batch, self.queries, self.heads, self.world = 256, coords.shape[0], 3, world
        g = torch.Generator(device=device).manual_seed(seed)
        self.grid = torch.randn(self.batch, self.queries, self.heads, 4, 12, device=device, generator=g)
        self.out = torch.empty(self.batch, self.heads, self.queries, self.queries, device=device)
        self.grad_out = torch.randn(self.out.shape, device=device, generator=g)
        self.device = device

    @property
    def bytes(self) -> float:  # grid read + bias written + the seven (Q, Q) tables read once
        q = self.queries
        return 4.0 * (self.grid.numel() + self.out.numel()) + q * q * (4 * 8 + 2 * 4 + 1)

    @property
    def backward_bytes(self) -> float:  # grad_out read + grad_grid written + tables
        q = self.queries
        return 4.0 * (self.grad_out.numel() + self.grid.numel()) + q * q * (4 * 8 + 2 * 4 + 1)

    @property
    def units_per_step(self) -> float:
        return self.bytes * self.world / 1e9

    @property
    def config(self) -> dict:
        return {"workload": f"dense_look_grid: grid ({self.batch}, {self.queries}, {self.heads}, 4, 12) fp32 -> "
                            f"bias ({self.batch}, {self.heads}, {self.queries}, {self.queries}) fp32, "
                            "14x14 hex lattice tables", "batch": self.batch, "heads": self.heads,
                "queries": self.queries}

    def step(self):
        from intp_preliminary_b200 import dense_look_grid_forward

        dense_look_grid_forward(self.grid, *self.tables, out=self.out)

    def backward_step(self):
        from intp_preliminary_b200 import dense_look_grid_backward

        dense_look_grid_backward(self.grad_out, *self.tables, grid_shape=self.grid.shape)

    def e2e_inputs(self):
        return [self.grid.cpu().pin_memory()]

    def e2e_output(self):
        return torch.empty(self.out.shape, dtype=self.out.dtype).pin_memory()

    def e2e_step(self, host_inputs, host_out):
        from intp_preliminary_b200 import dense_look_grid_sample

        grid = host_inputs[0].to(self.device, non_blocking=True)
        host_out.copy_(dense_look_grid_sample(grid, *self.tables), non_blocking=True)

    def cpu_reference(self):
        from oracle.dense_look_grid import dense_look_grid_np

        batch = 8
        grid = self.grid[:batch].cpu().numpy()
        tables = {name: t.cpu().numpy() for name, t in zip(
            ("radial0", "radial1", "angular0", "angular1", "radial_fraction", "angular_fraction", "valid"),
            self.tables)}
        dense_look_grid_np(grid, tables)
        times, t_end = [], time.perf_counter() + 10.0
        while time.perf_counter() < t_end or len(times) < 3:
            t0 = time.perf_counter()
            dense_look_grid_np(grid, tables)
            times.append(time.perf_counter() - t0)
        sample_bytes = self.bytes * batch / self.batch
        return sample_bytes / statistics.median(times) / 1e9, \
            f"{batch} of {self.batch} images of dense_look_grid through the oracle sampler (numpy float64)"


# --------------------------------------------------------------------------- timing
def _model_attention_ms(work, args, ctx, flush: torch.Tensor) -> float:
    """Mean device ms of one Look-attention launch on the model's own inputs:
    the 12 layers' attention arguments from one eager forward, replayed as one
    CUDA graph (12 launches back to back, no host gaps), CUDA events around
    each replay and the L2 flushed before it."""
    from intp_preliminary_b200.look_attention import look_attention_forward
    from intp_preliminary_b200.sharding import max_over_ranks

    model = work.model
    inputs = []
    model.attention_inputs = inputs
    work.eager_step()
    model.attention_inputs = None
    outs = [torch.empty_like(q) for q, *_ in inputs]

    def launches():
        for (q, k, v, pose, fields, scale), out in zip(inputs, outs):
            look_attention_forward(q, k, v, pose, fields, scale=scale, out=out)

    launches()  # warm-up outside capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        launches()
    times = _timed_steps(graph.replay, args.steps, args.warmup, ctx, flush)
    del graph
    return max_over_ranks(statistics.mean(times), ctx) / len(inputs)


def _timed_steps(step, steps: int, warmup: int, ctx, flush: torch.Tensor) -> list[float]:
    from intp_preliminary_b200.sharding import barrier

    stream = torch.cuda.current_stream(ctx.device)
    for _ in range(warmup):
        step()
    torch.cuda.synchronize(ctx.device)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    barrier(ctx)
    torch.cuda.synchronize(ctx.device)
    for i in range(steps):
        flush.fill_(i & 0xFF)  # 256 MiB write: evicts inputs from the 126 MB L2
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize(ctx.device)
    barrier(ctx)
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


def _look_roofline(flops: float, per_launch_ms: float, peaks: dict, traffic, kernel: str, where: str) -> dict:
    achieved = flops / (per_launch_ms * 1e-3) / 1e12
    return {"bound": "tensor", "achieved": round(achieved, 2), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
            "frac": round(achieved / peaks["bf16_tflops"], 4),
            "peak_source": f"{peaks['source']} bf16 dense (burst)", "traffic": traffic, "kernel": kernel,
            "launch_ms": round(per_launch_ms, 5), "where": where}


def _model_attention_roofline(batch: int, per_launch_ms: float, peaks: dict, traffic, where: str) -> dict:
    """The Look attention on the model's inputs (B x 3 heads x 196 tokens, D 64).

    Its arithmetic intensity, 4*B*H*N^2*D FLOPs over the algorithmic bytes
    (q, k, v and the output in bf16, the (B, 195, 3, 12) fp32 Look pose), is
    about 90 FLOP/byte: below the measured ridge point (bf16 peak / HBM
    bandwidth, about 251 FLOP/byte), so HBM is the roof.  The tensor-core
    fraction is reported beside it."""
    flops = 4.0 * batch * 3 * 196 * 196 * 64
    algo_bytes = 3 * batch * 3 * 196 * 64 * 2 + batch * 195 * 3 * 12 * 4 + batch * 3 * 196 * 64 * 2
    sec = per_launch_ms * 1e-3
    gbs, tflops = algo_bytes / sec / 1e9, flops / sec / 1e12
    ridge = peaks["bf16_tflops"] * 1e12 / (peaks["hbm_gbs"] * 1e9)
    return {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(gbs / peaks["hbm_gbs"], 4), "traffic": traffic, "kernel": "sla_short_kernel",
            "peak_source": f"{peaks['source']} HBM copy bandwidth", "launch_ms": round(per_launch_ms, 5),
            "algorithmic_bytes": algo_bytes, "flops": flops,
            "intensity_flop_per_byte": round(flops / algo_bytes, 1), "ridge_flop_per_byte": round(ridge, 1),
            "tensor_achieved_tflops": round(tflops, 2), "tensor_frac": round(tflops / peaks["bf16_tflops"], 4),
            "where": where}


def _nl1_roofline(work, per_launch_ms: float, peaks: dict) -> dict:
    """negative-L1: GB/s against HBM as asked, and beside it the op rate
    against the FP32 lanes' rate at the maximum SM clock (148 SMs x 128
    lanes; one lane-op per counted op) - the kernel is FP32-pipe bound."""
    gbs = work.bytes / (per_launch_ms * 1e-3) / 1e9
    fp32_peak = 148 * 128 * 1.965e9 / 1e12
    tops = work.flops / (per_launch_ms * 1e-3) / 1e12
    return {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(gbs / peaks["hbm_gbs"], 4), "traffic": NL1_TRAFFIC_BYTES.get(work.features),
            "kernel": "nl1_vec_kernel", "peak_source": f"{peaks['source']} HBM copy bandwidth",
            "launch_ms": round(per_launch_ms, 5),
            "note": "FP32-pipe bound; fp32_tops / fp32_peak_tops is the binding fraction",
            "fp32_tops": round(tops, 2), "fp32_peak_tops": round(fp32_peak, 1), "fp32_frac": round(tops / fp32_peak, 4)}


def _side_line(work, args, ctx, flush, roofline_fn) -> dict:
    """Device rate, roofline, end-to-end rate and CPU baseline of a workload
    timed beside the model (the same timing rules as the main line)."""
    from intp_preliminary_b200.sharding import max_over_ranks

    steps = max(args.steps, 5)
    times = _timed_steps(work.step, steps, args.warmup, ctx, flush)
    ms = max_over_ranks(statistics.mean(times), ctx)
    line = {"config": work.config, "metric": work.metric, "unit": work.unit,
            "value": round(work.units_per_step / (ms * 1e-3), 4), "ms_per_step": round(ms, 5),
            "roofline": roofline_fn(ms)}
    host_inputs, host_out = work.e2e_inputs(), work.e2e_output()
    e2e_times = _timed_steps(lambda: work.e2e_step(host_inputs, host_out), steps, args.warmup, ctx, flush)
    e2e_ms = max_over_ranks(statistics.mean(e2e_times), ctx)
    line["e2e"] = {"value": round(work.units_per_step / (e2e_ms * 1e-3), 4), "unit": work.unit,
                   "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in host_inputs),
                   "d2h_bytes_per_step": host_out.numel() * host_out.element_size()}
    if ctx.is_main and not args.no_cpu_baseline:
        result = work.cpu_reference()
        line["cpu_baseline"] = {"value": round(result[0], 6), "unit": work.unit, "cores": torch.get_num_threads(),
                                "kind": result[2] if len(result) > 2 else "port", "sample": result[1]}
    return line


def _reference_model_line(args, ctx, flush):
    """`bench.py --workload reference_model` (the reference's own half6d3r
    model code from baseline/_ref, unchanged, on this package's operators) in a
    child process - its imports replace the reference's operator modules, which
    this process's CPU baseline still needs.  One GPU runs only."""
    if ctx.world != 1 or not (REFERENCE_DIR / "model" / "deit_tiny_rot_hex_look.py").exists():
        return None
    cmd = [sys.executable, str(ROOT / "bench.py"), "--workload", "reference_model", "--steps", str(max(args.steps, 5)),
           "--warmup", str(args.warmup), "--no-cpu-baseline"]
    run = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    lines = [l for l in run.stdout.splitlines() if l.startswith("{")]
    if run.returncode != 0 or not lines:
        return {"unavailable": f"reference_model run failed (rc {run.returncode})"}
    child = json.loads(lines[-1])
    return {key: child[key] for key in ("metric", "value", "unit", "ms_per_step", "config", "e2e", "clocks",
                                         "look_registry_hits_per_step") if key in child}


def run_ours(args) -> None:
    from intp_preliminary_b200 import check_device_status
    from intp_preliminary_b200.sharding import barrier, init_from_env, max_over_ranks, shutdown

    ctx = init_from_env("nccl")
    if ctx.world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={ctx.world}; launch N>1 with torchrun")
    device = ctx.device
    peaks = _peaks()
    scaling = "weak"
    per_gpu = args.batch
    if args.global_batch is not None:
        if args.global_batch % ctx.world:
            raise SystemExit(f"--global-batch {args.global_batch} does not split over {ctx.world} GPUs")
        per_gpu, scaling = args.global_batch // ctx.world, "strong"
    if args.workload == "model":
        work = ModelWorkload(ctx, per_gpu, seed=1234)
    elif args.workload == "reference_model":
        work = ReferenceModelWorkload(ctx, per_gpu, seed=1234)
    elif args.workload.startswith("look"):
        work = LookWorkload(args.workload, device, seed=1234 + ctx.rank, world=ctx.world)
    elif args.workload == "dense_look_grid":
        work = DenseLookGridWorkload(device, seed=1234 + ctx.rank, world=ctx.world)
    else:
        work = NegativeL1Workload(device, seed=1234 + ctx.rank, world=ctx.world, features=args.features)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    visible = [v for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    gpu_index = visible[ctx.local_rank] if ctx.local_rank < len(visible) else str(ctx.local_rank)

    with ClockSampler(gpu_index) as clocks:
        times = _timed_steps(work.step, args.steps, args.warmup, ctx, flush)
    check_device_status(device)
    total_ms = max_over_ranks(sum(times), ctx)
    ms_per_step = total_ms / args.steps
    value = work.units_per_step * args.steps / (total_ms * 1e-3)
    per_launch_ms = statistics.mean(times)

    extra = {}
    if isinstance(work, ReferenceModelWorkload):
        from intp_preliminary_b200.look_registry import REGISTRY

        hits = REGISTRY.hits
        work.step()
        torch.cuda.synchronize(device)
        roofline = None
        launches = 12 * args.steps  # this package's: the 12 attention launches (the rest is the reference's PyTorch)
        extra["look_registry_hits_per_step"] = REGISTRY.hits - hits
    elif isinstance(work, ModelWorkload):
        # The attention kernel on the model's own inputs: the 12 layers' attention
        # arguments of one forward, replayed as one CUDA graph of 12 launches
        # (no host gaps), CUDA events around each replay, L2 flushed before it.
        attn_ms = _model_attention_ms(work, args, ctx, flush)
        roofline = _model_attention_roofline(
            work.batch, attn_ms, peaks, MODEL_ATTN_TRAFFIC_BYTES if work.batch == 256 else None,
            f"Look attention on the model forward's inputs (B{work.batch} H3 N196 D64 bf16, 68 slots, SLOT_FIELDS), "
            "the 12 layers' launches replayed as one CUDA graph, per launch")
        # ours per step: hex gather + post-GEMM + the first LayerNorm, then per block
        # qkv, Look attention, proj + residual + LN, fc1 + GELU, fc2 + residual + LN
        # (the tokenizer GEMM and the classifier head are cuBLAS)
        launches = (3 + 12 * 5) * args.steps
        # The other workloads of the hot path, each with its own device rate,
        # roofline, end-to-end rate (host buffers) and CPU baseline: the
        # long-sequence Look layer (B64 H6 N1025 bf16), the B8 H3 N197 fp32
        # Look layer, the standalone negative-L1 projection, and the
        # reference's own model code on this package's operators.
        if not args.no_side:
            cfg4 = LookWorkload("look_cfg4", device, seed=99 + ctx.rank, world=ctx.world)
            extra["look_attention_cfg4"] = _side_line(
                cfg4, args, ctx, flush, lambda ms: _look_roofline(
                    cfg4.flops, ms, peaks, CFG4_TRAFFIC_BYTES, "sla_tc_kernel",
                    "B64 H6 N1025 Look layer timed alone, one launch per step"))
            cfg1 = LookWorkload("look_cfg1", device, seed=98 + ctx.rank, world=ctx.world)
            extra["look_attention_cfg1"] = _side_line(
                cfg1, args, ctx, flush, lambda ms: {
                    **_look_roofline(cfg1.flops, ms, peaks, None, "sla_simt_kernel",
                                     "B8 H3 N197 fp32 Look layer timed alone (CUDA-core fp32 kernel)"),
                    "note": "fp32 correctness path on CUDA cores; the bf16 tensor peak is context only"})
            nl1 = NegativeL1Workload(device, seed=97 + ctx.rank, world=ctx.world)
            extra["negative_l1"] = _side_line(nl1, args, ctx, flush, lambda ms: _nl1_roofline(nl1, ms, peaks))
            if ctx.is_main:
                torch.cuda.synchronize(device)
                ref_model = _reference_model_line(args, ctx, flush)
                if ref_model is not None:
                    extra["reference_model"] = ref_model
        extra["model_flops_per_image"] = MODEL_FLOPS_PER_IMAGE
        extra["model_tflops"] = round(value * MODEL_FLOPS_PER_IMAGE / 1e12, 2)
    elif isinstance(work, LookWorkload):
        roofline = _look_roofline(work.flops, per_launch_ms, peaks,
                                  CFG4_TRAFFIC_BYTES if work.name == "look_cfg4" else None,
                                  "sla_tc_kernel" if work.dtype != torch.float32 else "sla_simt_kernel",
                                  "one launch per timed step")
        launches = args.steps
        # the backward on the same inputs: the tensor-core pass (16-bit inputs)
        # and the CUDA-core backward (delta, rows and cols kernels)
        work.backward_prepare(77 + ctx.rank)
        kinds = (("backward", "auto"), ("backward_cuda_cores", "simt")) if work.dtype != torch.float32 else \
            (("backward", "simt"),)
        for key, kind in kinds:
            bwd_ms = max_over_ranks(statistics.mean(_timed_steps(lambda: work.backward_step(kind), args.steps,
                                                                 args.warmup, ctx, flush)), ctx)
            bwd_tflops = work.backward_flops / (bwd_ms * 1e-3) / 1e12
            kernels = ("sla_bwd_dq_kernel + sla_bwd_dkdv_kernel (tcgen05; S, P, dP and dS recomputed "
                       "on chip, dQ / dK / dV and the slot gradient accumulated in TMEM)" if kind == "auto" else
                       "delta_kernel + rows_kernel + cols_kernel (CUDA cores, fp32 accumulation)")
            extra[key] = {"kernels": kernels, "ms": round(bwd_ms, 4), "tflops": round(bwd_tflops, 3),
                          "flops": "algorithmic 10*B*H*N^2*D",
                          "frac_of_bf16_peak": round(bwd_tflops / peaks["bf16_tflops"], 4)}
    elif isinstance(work, DenseLookGridWorkload):
        gbs = work.bytes / (per_launch_ms * 1e-3) / 1e9
        roofline = {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": round(gbs / peaks["hbm_gbs"], 4), "traffic": None, "kernel": "dlg_forward_kernel",
                    "peak_source": f"{peaks['source']} HBM copy bandwidth"}
        bwd_times = _timed_steps(work.backward_step, args.steps, args.warmup, ctx, flush)
        bwd_ms = max_over_ranks(statistics.mean(bwd_times), ctx)
        bwd_gbs = work.backward_bytes / (bwd_ms * 1e-3) / 1e9
        extra["backward"] = {"kernel": "dlg_backward_kernel", "ms": round(bwd_ms, 4), "achieved_gbs": round(bwd_gbs, 1),
                             "frac": round(bwd_gbs / peaks["hbm_gbs"], 4)}
        launches = args.steps
    else:
        gbs = work.bytes / (per_launch_ms * 1e-3) / 1e9
        roofline = _nl1_roofline(work, per_launch_ms, peaks)
        launches = args.steps
        work.backward_prepare(77 + ctx.rank)
        bwd_ms = max_over_ranks(statistics.mean(_timed_steps(work.backward_step, args.steps, args.warmup, ctx,
                                                             flush)), ctx)
        extra["backward"] = {"kernels": "nl1_sign_kernel x 2 (grad_x, grad_w)", "ms": round(bwd_ms, 4),
                             "fp32_tops": round(2 * work.flops / (bwd_ms * 1e-3) / 1e12, 2),
                             "ops": "2 x 2*M*P*F (sign and multiply-add, both gradients)"}

    # End-to-end through the public API with pinned host buffers.
    host_inputs = work.e2e_inputs()
    host_out = work.e2e_output()
    if isinstance(work, ReferenceModelWorkload):
        e2e_times = _timed_steps(lambda: work.e2e_step(host_inputs, host_out), args.steps, args.warmup, ctx, flush)
        e2e_total = max_over_ranks(sum(e2e_times), ctx)
        h2d = host_inputs[0].numel() * host_inputs[0].element_size()
    elif isinstance(work, ModelWorkload):
        # Batches stream from host memory (each step copies its own 154 MB
        # batch, larger than L2); copies overlap the previous step's forward.
        work.e2e_run(host_inputs, host_out, args.warmup)
        barrier(ctx)
        e2e_total = max_over_ranks(work.e2e_run(host_inputs, host_out, args.steps), ctx)
        h2d = host_inputs[0].numel() * host_inputs[0].element_size()
    else:
        e2e_times = _timed_steps(lambda: work.e2e_step(host_inputs, host_out), args.steps, args.warmup, ctx, flush)
        e2e_total = max_over_ranks(sum(e2e_times), ctx)
        h2d = sum(t.numel() * t.element_size() for t in host_inputs)
    e2e_value = work.units_per_step * args.steps / (e2e_total * 1e-3)
    d2h = host_out.numel() * host_out.element_size() if ctx.is_main else 0

    cpu = None
    if ctx.is_main and not args.no_cpu_baseline:
        result = work.cpu_reference()
        cpu_value, sample = result[:2]
        cpu = {"value": round(cpu_value, 6), "unit": work.unit, "cores": torch.get_num_threads(),
               "kind": result[2] if len(result) > 2 else "port", "sample": sample}
    if ctx.is_main:
        line = {
            "metric": work.metric, "value": round(value, 3), "unit": work.unit, "n_gpus": ctx.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": {torch.bfloat16: "bf16", torch.float32: "f32"}[work.dtype],
            "data": "synthetic (seeded N(0,1) images / q,k,v ~ N(0,1)/8, U(-1,1) Look fields; random-init weights)",
            "config": {**work.config,
                       "parallelism": f"batch-sharded replicas x{ctx.world} ({scaling}), logits gathered to rank 0"
                       if isinstance(work, ModelWorkload) else f"independent replicas x{ctx.world} (weak)",
                       "l2": "flushed between steps (256 MiB write outside the timed events)"},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 4), "unit": work.unit, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            "clocks": clocks.summary(),
            **extra,
        }
        print(json.dumps(line), flush=True)
    shutdown(ctx)


def run_reference(args) -> None:
    """The reference's CPU algorithm on bounded samples of the same workload (rank 0 only)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    kind = "port"
    if args.workload in ("model", "reference_model"):
        images = torch.randn(2, 3, 224, 224, generator=torch.Generator().manual_seed(1234))
        model = _reference_half6d3r(drop_in=False)
        if model is not None:
            def step():
                with torch.no_grad():
                    model(images)

            kind = "reference"
            sample = "2 images per step through the reference's own DeiTTinyRotHexLook (baseline/_ref) on CPU"
        else:
            from intp_preliminary_b200.share_vit import ShareViTHalf6d3r
            from oracle.share_vit_cpu import reference_forward_cpu

            port = ShareViTHalf6d3r(precision="fp32").init_weights(seed=0, look_grid_std=0.02)
            step = lambda: reference_forward_cpu(port, images)  # noqa: E731
            sample = "2 images per step through the reference CPU algorithm (oracle port: dense fields + explicit attention)"
        units, unit = 2.0, "images/s"
        metric = ReferenceModelWorkload.metric if args.workload == "reference_model" else ModelWorkload.metric
        per_gpu = args.global_batch // args.gpus if args.global_batch else args.batch
        config = {"workload": f"{args.workload}: half6d3r SHARE-ViT DeiT-Tiny forward, {per_gpu} images per GPU",
                  "batch_per_gpu": per_gpu}
        dtype = "f32"
    elif args.workload.startswith("look"):
        work = _CpuLook(args.workload)
        step, units, unit = work.step, work.sample_flops / 1e12, "TFLOP/s"
        metric, config, sample, dtype = LookWorkload.metric, work.config, work.sample, work.dtype_name
    elif args.workload == "negative_l1":
        from oracle.negative_l1 import negative_l1_torch

        g = torch.Generator().manual_seed(1234)
        rows, protos, features = 2048, 576, 1728
        x, w = torch.randn(rows, features, generator=g), torch.randn(protos, features, generator=g) * 0.5
        step = lambda: negative_l1_torch(x, w)  # noqa: E731
        units, unit = 2.0 * rows * protos * features / 1e12, "TFLOP/s"
        metric, dtype = NegativeL1Workload.metric, "f32"
        config = {"workload": f"negative_l1: x ({256 * 196}, {features}) fp32 vs prototypes ({protos}, {features})",
                  "rows": 256 * 196, "protos": protos, "features": features}
        sample = f"{rows} rows of negative_l1 per step, -cdist p=1"
    else:
        from intp_preliminary_b200 import hexgrid
        from oracle.dense_look_grid import dense_look_grid_np, sampling_tables_np

        tables = sampling_tables_np(hexgrid.offset_row_lattice(14, 14))
        grid = torch.randn(8, 196, 3, 4, 12, generator=torch.Generator().manual_seed(1234)).numpy()
        step = lambda: dense_look_grid_np(grid, tables)  # noqa: E731
        units = (4.0 * (grid.size + 8 * 3 * 196 * 196) + 196 * 196 * 41 * 8 / 256) / 1e9
        unit, metric, dtype = "GB/s", DenseLookGridWorkload.metric, "f32"
        config = {"workload": "dense_look_grid: grid (256, 196, 3, 4, 12) fp32 -> bias (256, 3, 196, 196) fp32, "
                              "14x14 hex lattice tables", "batch": 256, "heads": 3, "queries": 196}
        sample = "8 of 256 images of dense_look_grid per step through the oracle sampler (numpy float64)"
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        step()
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    value = units * len(times) / sum(times)
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": round(value, 6), "unit": unit, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * sum(times) / len(times), 3),
        "higher_is_better": True, "scaling": "strong" if args.global_batch else "weak", "vs_baseline": None,
        "dtype": dtype, "data": "synthetic", "config": config,
        "cpu_baseline": {"value": round(value, 6), "unit": unit, "cores": torch.get_num_threads(), "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(value, 6), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


class _CpuLook:
    """The reference's CPU path (oracle port: one-hot fields einsum) on a bounded
    per-step sample of a Look workload: one (batch, head) slice per step."""

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
    parser.add_argument("--steps", type=int, default=10)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--workload", choices=["model", "reference_model", "look_cfg4", "look_cfg1", "negative_l1",
                                               "dense_look_grid"], default="model")
    parser.add_argument("--batch", type=int, default=256, help="images per GPU (model workloads, weak scaling)")
    parser.add_argument("--global-batch", type=int, default=None,
                        help="total images over all GPUs (model workloads, strong scaling)")
    parser.add_argument("--features", type=int, default=1728, help="negative_l1 feature size F")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-side", action="store_true",
                        help="model workload: skip the side lines (long Look layer, fp32 Look layer, "
                             "negative-L1, reference model code)")
    args = parser.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
