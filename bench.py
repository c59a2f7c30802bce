#!/usr/bin/env python
"""Benchmark of the log-space hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

One JSON line on rank 0.  Default workload (the headline metric): the batched
log-space contraction 'bik,bkj->bij', b=128, i=k=j=512, fp32 log-values drawn
N(0, 8^2) from seed 1, logspace_max mode — "log-space einsum TFLOP/s" over
algorithmic FLOPs (2*b*i*j*k per step).  A step is one pass of the hot path
over the whole batch: the row-shift pass over A, the column-shift pass over B
and the fused contraction kernel (the launches xe_logspace_gemm makes for this
shape); the same step with B prepared once is reported beside it.  The line also
carries the folded-circuit throughput (samples/s) of the 32x32 quad-tree
circuit, batch 8192 per GPU (--circuit-batch), as `secondary`, its training
step, the 8192^3 and 32768^3 contractions, the Tucker layer, the row softmax,
and the headline expression in the scaled_sum mode.

Multi-GPU (torchrun, one process per GPU, NCCL): most lines are weak-scaled
(every rank its own batch, no data-path collective; the circuit gathers its
per-sample log-likelihoods with one all_gather per step); the 32768^3
contraction is A row-sharded with B broadcast once, and the circuit is also
run as one batch sharded over the ranks (strong scaling).  Times are
CUDA-event times, the max over ranks.

``--impl reference`` times the reference package itself (extended_einsum,
installed unmodified into baseline/_ref by baseline/install_reference.sh) on
the host cores, rank 0 only, on the same workload: its public
``TensorExpression.materialize('logspace_max')``, which on torch compiles the
translated program with torch.compile (backends/torch.py:141-150; the one-time
compile is excluded), and beside it the eager ``run_program`` of the same
backend program (demo/cirkit.py:428-435).  The repo line's ``cpu_baseline``
is that same arm, run as a CUDA-free child process.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
REFERENCE_PACKAGE = ROOT / "baseline" / "_ref"
sys.path.insert(0, str(ROOT))

SPLIT_TF32_NOTE = "split-TF32 (3 TF32 products per multiply-add): peak = measured bf16 / 2 (TF32 rate) / 3"


# ---------------------------------------------------------------------------
# environment


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data.get("hbm_gbs", 6650.0), "bf16_tflops": data.get("bf16_tflops", 1590.0),
                "bf16_tflops_sustained": data.get("bf16_tflops_sustained", 1400.0), "basis": "of measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "basis": "of fallback"}


def profiled_traffic() -> dict:
    path = ROOT / "profiles" / "traffic.json"
    return json.loads(path.read_text()) if path.exists() else {}


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML during the timed region."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int) -> None:
        self.samples: list[int] = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            uuid = torch.cuda.get_device_properties(device_index).uuid
            handle = None
            for i in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                raw = pynvml.nvmlDeviceGetUUID(h)
                raw = raw.decode() if isinstance(raw, bytes) else raw
                if raw.replace("GPU-", "") == str(uuid):
                    handle = h
            self._handle = handle or pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self._nvml = None

    def _run(self) -> None:
        nv = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
            except Exception:  # noqa: BLE001
                break
            time.sleep(0.002)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def report(self) -> dict | None:
        if self._nvml is None or not self.samples:
            return None
        reasons = [name for bit, name in self.REASONS.items() if self.reasons & bit]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# workloads


class LogspaceBmm:
    """'bik,bkj->bij', b=128, i=k=j=512, N(0, 8^2) log-values, logspace_max."""

    metric = "log-space einsum TFLOP/s"
    unit = "TFLOP/s"
    batch, m, n, k = 128, 512, 512, 512
    launches_per_step = 3  # shift of A, shift of B, contraction kernel

    def __init__(self, device: torch.device, rank: int) -> None:
        gen = torch.Generator().manual_seed(1 + 1000 * rank)
        self.a_host = (8.0 * torch.randn(self.batch, self.m, self.k, generator=gen)).pin_memory()
        self.b_host = (8.0 * torch.randn(self.batch, self.k, self.n, generator=gen)).pin_memory()
        self.a = self.a_host.to(device)
        self.b = self.b_host.to(device)
        self.out_host = torch.empty(self.batch, self.m, self.n).pin_memory()
        self.device = device
        self.kernel_events: list[tuple[torch.cuda.Event, ...]] = []
        self.prepared_events: list[tuple[torch.cuda.Event, ...]] = []

    @property
    def flops_per_step(self) -> float:
        return 2.0 * self.batch * self.m * self.n * self.k

    @classmethod
    def config(cls) -> dict:
        return {
            "workload": "logspace einsum 'bik,bkj->bij' b=128 i=k=j=512, fp32 N(0,8^2) log-values seed 1, logspace_max",
            "global_batch": cls.batch, "seq_len": None, "parallelism": None,
            "l2": "inputs (268 MB) larger than L2 (126 MB); no flush",
        }

    def step(self, record: bool) -> None:
        """The row shifts of A, the column shifts of B, the contraction kernel: the three launches
        xe_logspace_gemm makes for this shape (four row tiles of A: B is transformed in the kernel)."""
        from extended_einsum_b200 import ops

        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)] if record else None
        if record:
            ev[0].record()
        sa = ops.logspace_shift(self.a, shift="max")
        if record:
            ev[1].record()
        sb = ops.logspace_shift(self.b.transpose(1, 2), shift="max")
        if record:
            ev[2].record()
        ops.logspace_gemm_shifted(self.a, self.b, sa, sb)
        if record:
            ev[3].record()
            self.kernel_events.append(tuple(ev))

    def step_prepared(self, record: bool) -> None:
        """The same contraction with B prepared once (xe_logspace_b_prepare: column shifts, exp and
        TF32 split laid out as the kernel's stages), the path xe_logspace_gemm takes from 8 row tiles."""
        from extended_einsum_b200 import ops

        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)] if record else None
        if record:
            ev[0].record()
        sa = ops.logspace_shift(self.a, shift="max")
        if record:
            ev[1].record()
        prepared = ops.PreparedB(self.b, shift="max")
        if record:
            ev[2].record()
        ops.logspace_gemm_prepared(self.a, prepared, sa)
        if record:
            ev[3].record()
            self.prepared_events.append(tuple(ev))

    def kernel_ms(self) -> float:
        return statistics.mean(ev[2].elapsed_time(ev[3]) for ev in self.kernel_events)

    @staticmethod
    def _breakdown(events, names) -> dict:
        return {name: round(statistics.mean(ev[i].elapsed_time(ev[i + 1]) for ev in events), 4)
                for i, name in enumerate(names)}

    def breakdown_ms(self) -> dict:
        """Mean device time of each of the step's three launches."""
        return self._breakdown(self.kernel_events, ("shift_a", "shift_b", "contraction"))

    def prepared_line(self, ms_per_step: float, peaks: dict) -> dict:
        parts = self._breakdown(self.prepared_events, ("shift_a", "prepare_b", "contraction"))
        achieved = self.flops_per_step / (parts["contraction"] * 1e-3) / 1e12
        return {
            "metric": "log-space einsum TFLOP/s with B prepared", "value": round(self.flops_per_step / (ms_per_step * 1e-3) / 1e12, 3),
            "unit": "TFLOP/s", "ms_per_step": round(ms_per_step, 5), "step_breakdown_ms": parts,
            "kernel_frac_of_split_tf32_peak": round(achieved / (peaks["bf16_tflops"] / 6.0), 4),
            "workload": "the headline contraction as row shifts of A + xe_logspace_b_prepare + xe_logspace_gemm_prepared: "
                        "the kernel runs faster, the preparation pass costs more than it saves at 4 row tiles",
        }

    def e2e_step(self) -> None:
        """Public API with host buffers: the batch streamed through H2D, the kernels and D2H in 16 chunks.

        The step is bound by PCIe: 268 MB in and 134 MB out take 5.1 ms even without any kernel
        (6.7 TFLOP/s-equivalent); 16 chunks of 8 batches keep the copy engines busiest (8 chunks
        leave a longer fill and drain, 32 add host work per chunk)."""
        import extended_einsum_b200 as xb
        from extended_einsum_b200.streaming import materialize_streamed

        def build(a, b):
            return xb.log(xb.einsum("bik,bkj->bij", xb.exp(xb.array(a)), xb.exp(xb.array(b))))

        materialize_streamed(build, [self.a_host, self.b_host], self.out_host, "logspace_max", chunks=16, device=self.device)

    def scaled_step(self) -> None:
        """The same expression lowered in the scaled_sum mode, inputs resident on the device."""
        import extended_einsum_b200 as xb

        if not hasattr(self, "_scaled_program"):
            expr = xb.log(xb.einsum("bik,bkj->bij", xb.exp(xb.array(self.a)), xb.exp(xb.array(self.b))))
            program, _ = xb.extract_program(expr, "scaled_sum")
            self._scaled_program = xb.lower(program)
        xb.run_program(self._scaled_program, [self.a, self.b])

    @property
    def e2e_bytes(self) -> tuple[int, int]:
        return self.a_host.numel() * 4 + self.b_host.numel() * 4, self.out_host.numel() * 4

    def roofline(self, kernel_ms: float, peaks: dict, traffic: dict) -> dict:
        peak = peaks["bf16_tflops"] / 2.0 / 3.0
        achieved = self.flops_per_step / (kernel_ms * 1e-3) / 1e12
        return {
            "bound": "tensor", "kernel": "xe::gemm::lse_gemm_kernel", "achieved": round(achieved, 2), "peak": round(peak, 1),
            "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": traffic.get("lse_bmm"),
            "peak_basis": f"{SPLIT_TF32_NOTE} ({peaks['basis']})", "kernel_ms": round(kernel_ms, 4),
        }


class Circuit:
    """32x32 quad-tree CP circuit, K=64, 256 states, batch 8192 per GPU, log-likelihood output."""

    metric = "circuit samples/s"
    unit = "samples/s"

    def __init__(self, device: torch.device, rank: int, batch: int = 8192) -> None:
        from extended_einsum_b200.circuit import CircuitForward, QuadTreeCircuit

        self.circuit = QuadTreeCircuit(32, 32, 64, 256)
        gen = torch.Generator().manual_seed(3)
        params = self.circuit.init_parameters(gen)
        self.params = params
        self.batch = batch
        pixel_gen = torch.Generator().manual_seed(3 + 1000 * rank)
        self.pixels_host = torch.randint(256, (batch, self.circuit.variables), generator=pixel_gen, dtype=torch.uint8).pin_memory()
        self.pixels = self.pixels_host.to(device)
        dev = {k: (v.to(device) if isinstance(v, torch.Tensor) else [t.to(device) for t in v]) for k, v in params.items()}
        self.forward = CircuitForward(self.circuit, dev)
        self.ll_host = torch.empty(batch, 1).pin_memory()
        self.device = device

    def capture(self) -> None:
        """The whole forward pass (every layer's kernels) as one CUDA graph over self.pixels.

        A replay launches every kernel again on the current contents of self.pixels; only the
        host-side launch work is saved.  Three eager passes first resolve the kernels' one-time
        set-up outside the capture."""
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(3):
                self.forward(self.pixels)
        torch.cuda.current_stream(self.device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.graph_ll = self.forward(self.pixels)

    def step(self) -> torch.Tensor:
        self.graph.replay()
        return self.graph_ll

    def e2e_step(self) -> None:
        # this step's pixels into the graph's input buffer, the pass, the log-likelihoods out
        self.pixels.copy_(self.pixels_host, non_blocking=True)
        self.graph.replay()
        self.ll_host.copy_(self.graph_ll, non_blocking=True)

    def launches_per_step(self) -> int:
        levels = len(self.circuit.fold_counts)
        return 2 + 2 * levels + 2


class CircuitTrain:
    """The demo's training step on the same circuit (demo/cirkit.py:698-708): forward pass,
    loss = -mean log-likelihood, loss.backward() through the kernels' backward passes, an Adam
    step on the logits; with several ranks the gradients are averaged with one all_reduce per
    parameter (data parallel)."""

    def __init__(self, device: torch.device, rank: int, batch: int = 8192) -> None:
        from extended_einsum_b200.circuit import CircuitForward, QuadTreeCircuit

        self.circuit = QuadTreeCircuit(32, 32, 64, 256)
        gen = torch.Generator().manual_seed(3)
        params = self.circuit.init_parameters(gen)
        self.leaves = [params["categorical"].to(device).requires_grad_(),
                       *[t.to(device).requires_grad_() for t in params["levels"]],
                       params["root"].to(device).requires_grad_()]
        dev = {"categorical": self.leaves[0], "levels": self.leaves[1:-1], "root": self.leaves[-1],
               "var_of_fold": params["var_of_fold"].to(device)}
        self.forward = CircuitForward(self.circuit, dev)
        pixel_gen = torch.Generator().manual_seed(3 + 1000 * rank)
        self.pixels = torch.randint(256, (batch, self.circuit.variables), generator=pixel_gen, dtype=torch.uint8).to(device)
        self.batch = batch
        # Adam's fused CUDA step (one launch over every parameter; the same update as the default)
        self.opt = torch.optim.Adam(self.leaves, lr=1e-2, fused=True)

    def step(self, dist_on: bool) -> None:
        self.opt.zero_grad(set_to_none=True)
        loss = -self.forward(self.pixels).mean()
        loss.backward()
        if dist_on:
            world_size = torch.distributed.get_world_size()
            for p in self.leaves:
                torch.distributed.all_reduce(p.grad)
                p.grad.div_(world_size)
        self.opt.step()


class LoweredCircuit:
    """The same 32x32 circuit as the reference's own folded program, run through lower() / run_program.

    The program is the one demo/cirkit.py:466-479 builds: the demo's expression, folded by the
    reference's FoldSameShapedOperations and OptimizeContractionPaths (reference package from
    baseline/_ref).  Its data input is the (variables, batch, K) categorical probabilities that the
    demo gathers outside xe (demo/cirkit.py:525-527); here seeded softmax values stand in for them,
    resident on the device.  lower() fuses each level's Hadamard product into the next sum layer.
    """

    def __init__(self, device: torch.device, rank: int, batch: int, layer: str = "cp", side: int = 32,
                 units: int = 64) -> None:
        if str(REFERENCE_PACKAGE) not in sys.path:
            sys.path.insert(0, str(REFERENCE_PACKAGE))
        import extended_einsum as xe

        import extended_einsum_b200 as xb
        from extended_einsum_b200.circuit import demo_circuit_inputs, demo_circuit_program

        self.batch = batch
        program, data_input = demo_circuit_program(xe, side, side, units, batch, layer=layer)
        gen = torch.Generator(device=device).manual_seed(3 + 1000 * rank)
        self.inputs = demo_circuit_inputs(program, data_input, gen, device)
        self.lowered = xb.lower(program)
        self.run = xb.run_program
        self.launches = sum(1 for c in self.lowered.backend_calls if getattr(c, "fn", None) is not None and
                            getattr(getattr(c, "fn"), "__name__", "") != "<lambda>")

    def step(self, record: bool) -> torch.Tensor:
        return self.run(self.lowered, self.inputs)

    @staticmethod
    def tucker_flops_per_sample(variables: int, units: int) -> int:
        """2*O*I*J per layer fold (the fused (i,j) form), every level, the root's one output."""
        folds, f = 0, variables // 2
        while f >= 2:
            folds += f
            f //= 2
        return 2 * units**3 * folds + 2 * units * units

    @staticmethod
    def hbm_bytes_per_sample(variables: int = 1024, units: int = 64) -> int:
        """Layer-by-layer bytes per sample: the data rows read once, each level written once and read
        once by the next (its Hadamard product fused), the root's two rows read, one value written."""
        folds, f = 0, variables // 2
        while f >= 2:
            folds += f
            f //= 2
        return 4 * units * (2 * variables + 3 * folds + 2) + 4


# ---------------------------------------------------------------------------


def time_region(fn, steps: int, warmup: int, dist_on: bool) -> float:
    for _ in range(warmup):
        fn(False)
    torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn(True)
    end.record()
    end.synchronize()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    if dist_on:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
        torch.distributed.barrier()
    return ms


def large_matmul_step(a: torch.Tensor, b: torch.Tensor):
    """One 8192^3 log-space contraction 'ik,kj->ij' (shifts + kernel)."""
    from extended_einsum_b200 import ops

    def step(record: bool) -> None:
        ops.logspace_gemm(a, b)

    return step


def run_ours(args, rank: int, world: int, device: torch.device, dist_on: bool) -> dict | None:
    """Every workload of the line (``--only`` selects one: a profiling run, not the bench line)."""
    from extended_einsum_b200 import _lib
    from extended_einsum_b200 import distributed as xd
    from extended_einsum_b200 import ops

    _lib.load()
    peaks = measured_peaks()

    def want(name: str) -> bool:
        return args.only in (None, name)

    line: dict = {}
    if want("headline"):
        work = LogspaceBmm(device, rank)
        # the headline (device-resident) measurement
        sampler = ClockSampler(device.index or 0)
        with sampler:
            ms = time_region(work.step, args.steps, args.warmup, dist_on)
        kernel_ms = work.kernel_ms()
        if dist_on:
            t = torch.tensor([kernel_ms], device="cuda")
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            kernel_ms = float(t.item())
        ms_per_step = ms / args.steps
        value = world * work.flops_per_step / (ms_per_step * 1e-3) / 1e12
        line.update({
            "metric": work.metric, "value": round(value, 3), "unit": work.unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32 (split-TF32 tensor-core products, fp32 accumulation)", "data": "synthetic",
            "config": {**work.config(), "parallelism": f"batch-sharded x{world} (weak)"},
            "gpu_launches": work.launches_per_step * args.steps,
            "roofline": work.roofline(kernel_ms, peaks, profiled_traffic()),
            "step_breakdown_ms": work.breakdown_ms(),
            "clocks": sampler.report(),
        })
        p_ms = time_region(work.step_prepared, args.steps, args.warmup, dist_on) / args.steps
        line["prepared_b"] = work.prepared_line(p_ms, peaks)
    if want("e2e"):
        work = work if want("headline") else LogspaceBmm(device, rank)
        # end to end through the public API with host buffers
        e2e_steps = max(5, args.steps // 4)
        e2e_ms = time_region(lambda record: work.e2e_step(), e2e_steps, 3, dist_on) / e2e_steps
        h2d, d2h = work.e2e_bytes
        line["e2e"] = {"value": round(world * work.flops_per_step / (e2e_ms * 1e-3) / 1e12, 3), "unit": work.unit,
                       "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}
    if want("scaled"):
        work = work if (want("headline") or want("e2e")) else LogspaceBmm(device, rank)
        # the same contraction in the scaled_sum mode (device-resident inputs, lowered program)
        steps = max(3, args.steps // 2)
        scaled_ms = time_region(lambda record: work.scaled_step(), steps, 3, dist_on) / steps
        line["scaled_sum"] = {
            "metric": "log-space einsum TFLOP/s, scaled_sum mode",
            "value": round(world * work.flops_per_step / (scaled_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
            "ms_per_step": round(scaled_ms, 4),
            "workload": "the headline expression log(einsum(exp(A), exp(B))) materialized in scaled_sum (lowered: "
                        "one log-space contraction with the exp rule's shifts)",
        }
    work = None
    torch.cuda.empty_cache()

    if want("large"):
        # the 8192^3 contraction (per GPU, weak), log(U(0,1)) values
        gen = torch.Generator(device=device).manual_seed(4 + 1000 * rank)
        big_a = torch.log(torch.rand(1, 8192, 8192, device=device, generator=gen))
        big_b = torch.log(torch.rand(1, 8192, 8192, device=device, generator=gen))
        big_ms = time_region(large_matmul_step(big_a, big_b), 5, 3, dist_on) / 5
        big_value = world * 2.0 * 8192**3 / (big_ms * 1e-3) / 1e12
        del big_a, big_b
        line["large_8192"] = {
            "metric": "log-space einsum TFLOP/s, 'ik,kj->ij' 8192^3 per GPU", "value": round(big_value, 2), "unit": "TFLOP/s",
            "ms_per_step": round(big_ms, 3), "frac_of_split_tf32_peak": round(big_value / world / (peaks["bf16_tflops"] / 6.0), 4),
            "workload": "A, B = log(U(0,1)) 8192x8192 fp32, logspace_max, xe_logspace_gemm (row shifts, B prepared, kernel)",
        }
        torch.cuda.empty_cache()

    tgen = torch.Generator(device=device).manual_seed(2 + 1000 * rank)
    if want("tucker"):
        # the Tucker layer 'bfi,bfj,foij->bfo' (b=512, f=2048, i=j=o=32), linear softmax weights
        t_l = torch.randn(512, 2048, 32, device=device, generator=tgen) - 3.0
        t_r = torch.randn(512, 2048, 32, device=device, generator=tgen) - 3.0
        t_w = ops.softmax(torch.randn(2048, 32, 32, 32, device=device, generator=tgen), (2, 3))
        tucker_ms = time_region(lambda record: ops.logspace_tucker(t_l, t_r, t_w), 8, 3, dist_on) / 8
        tucker_value = world * 2.0 * 512 * 2048 * 32**3 / (tucker_ms * 1e-3) / 1e12
        del t_l, t_r, t_w
        line["tucker"] = {
            "metric": "log-space Tucker layer TFLOP/s", "value": round(tucker_value, 2), "unit": "TFLOP/s",
            "ms_per_step": round(tucker_ms, 4), "frac_of_split_tf32_peak": round(tucker_value / world / (peaks["bf16_tflops"] / 6.0), 4),
            "workload": "'bfi,bfj,foij->bfo' b=512 f=2048 i=j=o=32, l, r = N(-3,1), w = softmax of N(0,1) logits over (i,j), logspace_max",
            "flops_basis": "2*b*f*o*i*j, the fused (i,j) form; the kernel contracts j first on the tensor cores and i in "
                           "its epilogue, executing half of that as tensor work",
        }
    if want("softmax"):
        # row softmax of a (65536, 32768) matrix, 2 N(0,1)
        s_x = 2.0 * torch.randn(args.softmax_rows, 32768, device=device, generator=tgen)
        softmax_ms = time_region(lambda record: ops.softmax(s_x, 1), 5, 3, dist_on) / 5
        softmax_gbs = 2 * s_x.numel() * 4 / (softmax_ms * 1e-3) / 1e9
        del s_x
        torch.cuda.empty_cache()
        line["softmax"] = {
            "metric": "softmax GB/s (one read and one write of the matrix)", "value": round(world * softmax_gbs, 1), "unit": "GB/s",
            "ms_per_step": round(softmax_ms, 4), "hbm_frac": round(softmax_gbs / peaks["hbm_gbs"], 4),
            "workload": f"row softmax of a ({args.softmax_rows}, 32768) fp32 matrix of 2 N(0,1) values",
        }
    if want("huge"):
        # the 32768^3 contraction 'ik,kj->ij', log(U(0,1)) values: A row-sharded over the ranks, B
        # broadcast once from rank 0 (NCCL), every rank contracting its rows with the full B
        # (strong scaling: the whole contraction is the work at every N)
        size = 32768
        lo, hi = xd.shard_bounds(size, rank, world)
        a_rows = torch.log(torch.rand(hi - lo, size, device=device, generator=tgen))
        bgen = torch.Generator(device=device).manual_seed(4)
        b_full = torch.log(torch.rand(size, size, device=device, generator=bgen)) if rank == 0 else None
        mm = xd.RowShardedMatmul(shift="max")
        torch.cuda.synchronize()
        bc0, bc1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        bc0.record()
        mm.set_b(b_full, (size, size), src=0, device=device)
        bc1.record()
        torch.cuda.synchronize()
        bcast_ms = bc0.elapsed_time(bc1)
        huge_ms = time_region(lambda record: mm(a_rows, size), 2, 1, dist_on) / 2
        if dist_on:
            t = torch.tensor([bcast_ms], device="cuda")
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            bcast_ms = float(t.item())
        huge_value = 2.0 * size**3 / (huge_ms * 1e-3) / 1e12
        del a_rows, b_full, mm
        torch.cuda.empty_cache()
        line["large_32768"] = {
            "metric": "log-space einsum TFLOP/s, 'ik,kj->ij' 32768^3, A row-sharded over the GPUs",
            "value": round(huge_value, 2), "unit": "TFLOP/s", "ms_per_step": round(huge_ms, 2), "scaling": "strong",
            "frac_of_split_tf32_peak": round(huge_value / world / (peaks["bf16_tflops"] / 6.0), 4),
            "frac_of_sustained_split_tf32_peak": round(
                huge_value / world / (peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]) / 6.0), 4),
            "b_broadcast_ms": round(bcast_ms, 2) if world > 1 else None,
            "workload": f"A, B = log(U(0,1)) 32768x32768 fp32, logspace_max; rank r owns {hi - lo} rows of A, B "
                        "broadcast once from rank 0 (ncclBroadcast of 4 GiB, timed apart), each step "
                        "xe_logspace_gemm of the rank's rows (row shifts, B prepared, kernel); 1 warm-up + 2 steps "
                        "(a long step: the sustained peak is its denominator)",
        }

    if want("circuit"):
        # secondary: the folded circuit, batch-sharded
        circ = Circuit(device, rank, args.circuit_batch)
        circ.capture()

        def circuit_step(record: bool) -> None:
            ll = circ.step()
            if dist_on:
                # batch-sharded: the per-sample log-likelihoods of all ranks, in rank order
                xd.gather_rows(ll, world * circ.batch)

        c_steps = max(3, args.steps // 2)
        c_ms = time_region(circuit_step, c_steps, max(3, args.warmup), dist_on) / c_steps
        c_e2e_ms = time_region(lambda record: circ.e2e_step(), max(3, c_steps // 2), 2, dist_on) / max(3, c_steps // 2)
        flops_sample = circ.circuit.flops_per_sample()
        state_table = circ.circuit.uses_state_table(circ.batch)
        bytes_sample = circ.circuit.hbm_bytes_per_sample(state_table)
        c_value = world * circ.batch / (c_ms * 1e-3)
        del circ
        torch.cuda.empty_cache()
        line["secondary"] = {
            "metric": "circuit samples/s", "value": round(c_value, 1), "unit": "samples/s",
            "workload": f"folded 32x32 quad-tree CP circuit, K=64, 256 states, batch {args.circuit_batch} per GPU, uint8 pixels seed 3, "
                        "each step a replay of the forward pass captured as one CUDA graph",
            "first_layer": "state table (F0 x 256 rows) + gathered Hadamard pairs" if state_table else "per sample, gather fused",
            "hbm_bytes_per_sample": bytes_sample,
            "ms_per_step": round(c_ms, 4),
            "hbm_frac": round(bytes_sample * c_value / world / 1e9 / peaks["hbm_gbs"], 4),
            "hbm_gbs_algorithmic": round(bytes_sample * c_value / world / 1e9, 1),
            "tflops_algorithmic": round(flops_sample * c_value / world / 1e12, 2),
            "e2e_samples_per_s": round(world * args.circuit_batch / (c_e2e_ms * 1e-3), 1),
        }

    if want("circuit"):
        # the training step (forward, backward, Adam), batch circuit_batch per GPU
        tr = CircuitTrain(device, rank, args.circuit_batch)
        tr_steps = max(3, args.steps // 10)
        tr_ms = time_region(lambda record: tr.step(dist_on), tr_steps, 3, dist_on) / tr_steps
        del tr
        torch.cuda.empty_cache()
        line["circuit_train"] = {
            "metric": "circuit training samples/s (forward + backward + Adam)", "value": round(world * args.circuit_batch / (tr_ms * 1e-3), 1),
            "unit": "samples/s", "ms_per_step": round(tr_ms, 3), "scaling": "weak",
            "workload": f"the folded 32x32 quad-tree CP circuit, batch {args.circuit_batch} per GPU: -mean log-likelihood, "
                        "loss.backward() through the fused layer backward kernels, torch.optim.Adam (fused) on the logits"
                        + ("; gradients averaged with one all_reduce per parameter" if dist_on else ""),
        }

    if want("circuit") and world > 1:
        # the same circuit strong-scaled: one batch of circuit_batch samples sharded over the ranks
        lo, hi = xd.shard_bounds(args.circuit_batch, rank, world)
        circ_s = Circuit(device, rank, hi - lo)
        circ_s.capture()

        def strong_step(record: bool) -> None:
            xd.gather_rows(circ_s.step(), args.circuit_batch)

        s_steps = max(3, args.steps // 2)
        s_ms = time_region(strong_step, s_steps, max(3, args.warmup), dist_on) / s_steps
        del circ_s
        torch.cuda.empty_cache()
        line["circuit_strong"] = {
            "metric": "circuit samples/s, one batch sharded over the GPUs", "value": round(args.circuit_batch / (s_ms * 1e-3), 1),
            "unit": "samples/s", "ms_per_step": round(s_ms, 4), "scaling": "strong",
            "workload": f"the folded 32x32 quad-tree CP circuit, {args.circuit_batch} samples in total, "
                        f"{hi - lo} per rank, log-likelihoods gathered with one all_gather per step",
        }

    # the reference's own folded circuit program through lower() / run_program (the drop-in path)
    if want("lowered") and (REFERENCE_PACKAGE / "extended_einsum").is_dir():
        low = LoweredCircuit(device, rank, args.circuit_batch)
        l_steps = max(3, args.steps // 4)
        l_ms = time_region(low.step, l_steps, 3, dist_on) / l_steps
        l_value = world * low.batch / (l_ms * 1e-3)
        l_bytes = LoweredCircuit.hbm_bytes_per_sample()
        lowered_line = {
            "metric": "circuit samples/s through lower()", "value": round(l_value, 1), "unit": "samples/s",
            "ms_per_step": round(l_ms, 4),
            "workload": f"the reference's folded program of the same circuit (its FoldSameShapedOperations + "
                        f"OptimizeContractionPaths), batch {low.batch} per GPU, data input (1024, batch, 64) "
                        "categorical probabilities resident, run_program of the lowered program, eager",
            "hbm_bytes_per_sample": l_bytes,
            "hbm_frac": round(l_bytes * l_value / world / 1e9 / peaks["hbm_gbs"], 4),
            "kernel_calls_per_step": low.launches,
        }
        del low
        torch.cuda.empty_cache()
        # the reference's folded Tucker circuit (--sum-product-layer tucker) over a 64x64 grid, K=32:
        # its first layer is the Tucker configuration b=512, f=2048, i=j=o=32
        tk = LoweredCircuit(device, rank, 512, layer="tucker", side=64, units=32)
        t_steps = max(3, args.steps // 4)
        t_ms = time_region(tk.step, t_steps, 3, dist_on) / t_steps
        t_flops = LoweredCircuit.tucker_flops_per_sample(4096, 32)
        lowered_line["tucker_circuit"] = {
            "metric": "Tucker circuit samples/s through lower()", "value": round(world * tk.batch / (t_ms * 1e-3), 1),
            "unit": "samples/s", "ms_per_step": round(t_ms, 4),
            "workload": "the reference's folded 64x64 quad-tree Tucker circuit (Kronecker + sum layers fused by "
                        "OptimizeContractionPaths into 'acde,abd,abe->abc'), K=32, batch 512 per GPU, data resident",
            "tflops_algorithmic": round(t_flops * tk.batch / (t_ms * 1e-3) / 1e12, 2),
            "frac_of_split_tf32_peak": round(t_flops * tk.batch / (t_ms * 1e-3) / 1e12 / (peaks["bf16_tflops"] / 6.0), 4),
            "kernel_calls_per_step": tk.launches,
        }
        del tk
        torch.cuda.empty_cache()
        line["circuit_lowered"] = lowered_line

    if rank != 0:
        return None
    if args.only is not None:
        line = {"only": args.only, **line}
    elif world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args)
    return line


def cpu_baseline(args) -> dict:
    """The reference arm below, run as a child process that never touches CUDA, with the same steps."""
    import subprocess

    env = {k: v for k, v in os.environ.items() if k not in ("OMP_NUM_THREADS", "MKL_NUM_THREADS")}
    cmd = [sys.executable, str(Path(__file__).resolve()), "--impl", "reference", "--steps", str(args.steps), "--warmup", str(args.warmup)]
    out = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=1800)
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    if out.returncode != 0 or not lines:
        return {"value": None, "unit": "TFLOP/s", "cores": None, "kind": "reference",
                "sample": f"reference arm failed (rc {out.returncode}): {out.stderr.strip().splitlines()[-1:] }"}
    ref = json.loads(lines[-1])
    base = dict(ref["cpu_baseline"])
    base["eager"] = ref.get("eager")
    return base


class ReferenceCPU:
    """The reference package's own CPU path on the headline workload (128 x 512^3, N(0, 8^2), seed 1).

    ``materialize`` is the reference's public call (interface/tensor_expression.py:104-117): extract
    the program, translate it with TorchBackendFunctions, compile it with TorchCompiler
    (torch.compile, backends/torch.py:141-150) and run it.  Later steps call the compiled
    ``_backend_code`` again, as a user re-running the materialized expression would; the compile is
    timed once and reported apart.  ``eager`` runs the same backend program through ``run_program``
    (backend_translation/runtime.py:9-21), the demo's path without --torch-compile.
    """

    def __init__(self) -> None:
        if not (REFERENCE_PACKAGE / "extended_einsum").is_dir():
            raise RuntimeError("the reference package is not installed in baseline/_ref (run baseline/install_reference.sh)")
        sys.path.insert(0, str(REFERENCE_PACKAGE))
        import extended_einsum as xe
        from extended_einsum.backend_translation.runtime import run_program
        from extended_einsum.backend_translation.translate import translate_to_backend_program
        from extended_einsum.backends.torch import TorchBackendFunctions

        gen = torch.Generator().manual_seed(1)
        a = 8.0 * torch.randn(LogspaceBmm.batch, LogspaceBmm.m, LogspaceBmm.k, generator=gen)
        b = 8.0 * torch.randn(LogspaceBmm.batch, LogspaceBmm.k, LogspaceBmm.n, generator=gen)
        self.expr = xe.log(xe.einsum("bik,bkj->bij", xe.exp(xe.array(a)), xe.exp(xe.array(b))))
        program, arguments = xe.extract_program(self.expr, "logspace_max")
        self.inputs = [arg.backend_array for arg in arguments]
        backend_program = translate_to_backend_program(program, TorchBackendFunctions())
        self.backend_calls = len(backend_program.backend_calls)
        self.eager = lambda: run_program(backend_program, self.inputs)
        self.compile_s = None

    def compiled(self):
        import torch._inductor.config as inductor_config

        # the image's CXX wrapper (/opt/gcc) lacks libgomp's specs, which inductor's OpenMP
        # CPU kernels need; the system g++ has them
        if os.path.exists("/usr/bin/g++"):
            inductor_config.cpp.cxx = (None, "/usr/bin/g++")
        t0 = time.perf_counter()
        self.expr.materialize("logspace_max")
        self.compile_s = time.perf_counter() - t0
        code = self.expr._backend_code
        inputs = [arg.backend_array for arg in self.expr._input_arguments]
        return lambda: code(inputs)


def time_cpu_steps(fn, steps: int, warmup: int, warm_s: float = 5.0) -> float:
    """Seconds per step over exactly `steps` calls, after `warmup` calls and at least `warm_s` s of calls.

    The first seconds of a fresh process run slower (the allocator's first large blocks are
    fresh pages), so warm-up runs until both bounds are met."""
    t0 = time.perf_counter()
    n = 0
    while n < warmup or time.perf_counter() - t0 < warm_s:
        fn()
        n += 1
    t0 = time.perf_counter()
    for _ in range(steps):
        fn()
    return (time.perf_counter() - t0) / steps


def run_reference(args, rank: int) -> dict | None:
    """The reference package's CPU path on the host cores, rank 0 only (same config as the repo line)."""
    if rank != 0:
        return None
    # every host thread this process may run on (the affinity set, not the machine's count)
    torch.set_num_threads(len(os.sched_getaffinity(0)) or 1)
    flops = 2.0 * LogspaceBmm.batch * LogspaceBmm.m * LogspaceBmm.n * LogspaceBmm.k
    ref = ReferenceCPU()
    kind, note = "compiled", None
    try:
        step = ref.compiled()
    except Exception as exc:  # noqa: BLE001 - torch.compile unusable on this host: the eager path is the anchor
        kind, note, step = "eager", f"torch.compile failed ({type(exc).__name__}); eager run_program is the anchor", ref.eager
    dt = time_cpu_steps(step, args.steps, args.warmup)
    value = flops / dt / 1e12
    eager_dt = dt if kind == "eager" else time_cpu_steps(ref.eager, max(3, args.steps // 2), 3)
    eager = {"value": round(flops / eager_dt / 1e12, 5), "unit": "TFLOP/s", "ms_per_step": round(eager_dt * 1e3, 2),
             "path": f"run_program of the translated backend program ({ref.backend_calls} torch calls)"}
    sample = (f"the whole workload per step (128 x 512^3), reference package from baseline/_ref, "
              f"{'materialize(): torch.compile of the translated program, compile excluded' if kind == 'compiled' else 'eager run_program'}")
    cores = torch.get_num_threads()
    world = args.gpus
    config = {**LogspaceBmm.config(), "parallelism": f"batch-sharded x{world} (weak)"}
    line = {
        "impl": "reference", "metric": LogspaceBmm.metric, "value": round(value, 5), "unit": LogspaceBmm.unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config,
        "cpu_baseline": {"value": round(value, 5), "unit": "TFLOP/s", "cores": cores, "kind": "reference", "sample": sample,
                         "path": kind, "host_cpus": os.cpu_count(),
                         "compile_s": None if ref.compile_s is None else round(ref.compile_s, 1)},
        "eager": eager,
        "e2e": {"value": round(value, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if note:
        line["note"] = note
    return line


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=50)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--circuit-batch", type=int, default=8192, help="circuit samples per GPU (default 8192)")
    parser.add_argument("--softmax-rows", type=int, default=65536, help="rows of the softmax workload (default 65536)")
    parser.add_argument("--only", choices=["headline", "e2e", "scaled", "large", "tucker", "softmax", "huge", "circuit",
                                           "lowered"], default=None,
                        help="run one workload alone (profiling; the line then carries that workload only)")
    args = parser.parse_args()
    if args.warmup < 3:
        parser.error("--warmup must be at least 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if world > 1:
            # torchrun pins every rank to one OpenMP thread; rank 0 times the CPU path in a
            # fresh process with the host's threads, the other ranks have nothing to do
            if rank == 0:
                env = {k: v for k, v in os.environ.items()
                       if k not in ("OMP_NUM_THREADS", "MKL_NUM_THREADS", "WORLD_SIZE", "RANK", "LOCAL_RANK",
                                    "LOCAL_WORLD_SIZE", "GROUP_RANK", "ROLE_RANK", "TORCHELASTIC_RUN_ID")}
                import subprocess

                subprocess.run([sys.executable, str(Path(__file__).resolve()), *sys.argv[1:]], env=env, check=True)
            return
        line = run_reference(args, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    dist_on = world > 1
    from extended_einsum_b200 import distributed as xd

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if dist_on:
        xd.init_distributed("nccl", timeout_s=120.0, device=device, nonblocking=False)
    try:
        line = run_ours(args, rank, world, device, dist_on)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if dist_on:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
