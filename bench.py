#!/usr/bin/env python3
"""Benchmark of the q6 image feed-forward MLP (one Qwen-Image MMDiT block's img_ff).

Workload (one step): x bf16 [3456, 3072] (1728 target + 1728 reference-image
tokens of a 576x768 edit) -> q6 fc1 3072->12288 (+bias, GELU-tanh) -> q6 fc2
12288->3072 (+bias), MLX affine 6-bit weights with group size 64, seeded
synthetic N(0,1) activations and N(0,0.02) weights (no checkpoint exists here).
4 * 3456 * 3072 * 12288 = 521.84 GFLOP per step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One process per GPU (torchrun for N > 1).  The MLP is token-sharded: every
rank runs its own 3456-token batch with replicated weights and no collective
on the data path (weak scaling); the job value is all ranks' FLOPs over the
slowest rank's device time.  Rank 0 prints one JSON line.

Beside the headline, the line carries the few-row linears (``gemv``), one
full Qwen-Image MMDiT block (``block``: 3456 image + 256 text tokens, all 14
linears q6, joint attention) and the 60-block stack (``stack``), split over the
ranks when N > 1 in every multi-GPU form (BLOCK_FORMS, ``--block-form``).

--impl reference times the reference's own q6 kernel source
(shardedit_mlx/q6_metal_mlp.py SOURCE_QMM_T, compiled for the host by
oracle/build_ref.py) on the host cores, on full 3456-token steps of the same
workload (as many as fit about 110 s, at least one).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

TOKENS, DIM, HIDDEN, GROUP = 3456, 3072, 12288, 64
FLOP_PER_STEP = 4 * TOKENS * DIM * HIDDEN  # two linears, 2*M*N*K each
METRIC = "q6 img-FF MLP TFLOP/s & % bf16 peak at M=3456; q6 GEMV HBM GB/s; block ms 1/2/4/8 GPU"
WORKLOAD = "fused image feed-forward MLP of one MMDiT block, q6 gs64 (3456 tokens, 3072->12288->3072)"
L2_BYTES = 126 * 2**20


def parse_args() -> argparse.Namespace:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the host-core baseline leg")
    ap.add_argument("--no-gemv", action="store_true", help="skip the skinny-M GEMV side measurement")
    ap.add_argument("--no-block", action="store_true", help="skip the full MMDiT block measurement")
    ap.add_argument("--no-sweep", action="store_true", help="skip the q6 linear shape / M / group-size sweep")
    ap.add_argument("--no-stack", action="store_true", help="skip the 60-block stack (config 5)")
    ap.add_argument("--only", choices=["block", "gemv", "sweep", "stack", "kernels"], default=None,
                    help="run one side measurement alone and print its JSON (for profiling runs)")
    ap.add_argument("--gemv-case", default=None,
                    help="comma-separated GEMV case names to run (default: all of GEMV_CASES)")
    ap.add_argument("--block-form", choices=["auto", *BLOCK_FORMS], default="auto",
                    help="multi-GPU form of the block and the stack: context-parallel rows with all-gathered keys "
                         "and values, a batch first split over rank groups (cp), or tensor-parallel heads / FF "
                         "columns with fused peer-memory (tp-peer) or NCCL (tp-nccl) collectives; auto: the measured "
                         "faster one (cp for a batch that splits over the GPUs; for one sample tp-peer at 2 GPUs, cp "
                         "from 4)")
    return ap.parse_args()


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "bf16_tflops": float(data["bf16_tflops"]),
                "bf16_tflops_sustained": float(data.get("bf16_tflops_sustained", data["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def profiled_traffic() -> dict:
    """Per-launch DRAM bytes of the dominant kernels from the committed ncu summary."""

    path = ROOT / "profiles" / "dram_traffic.json"
    if path.exists():
        try:
            return json.loads(path.read_text())
        except (OSError, ValueError):
            return {}
    return {}


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled through NVML from a
    background thread every ~2 ms while the timed region runs (read-only; no
    GPU setting is touched)."""

    REASONS = {
        "hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
        "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
        "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
        "sw_power_cap": "nvmlClocksEventReasonSwPowerCap",
        "hw_power_brake_slowdown": "nvmlClocksEventReasonHwPowerBrakeSlowdown",
    }

    def __init__(self, gpu_index: int, period_s: float = 0.002) -> None:
        self.gpu = gpu_index
        self.period = period_s
        self.samples: list[tuple[int, int, int]] = []
        self._stop = None
        self._thread = None
        self._nvml = None
        self._handle = None

    def _sample(self) -> None:
        nv = self._nvml
        sm = nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM)
        mx = nv.nvmlDeviceGetMaxClockInfo(self._handle, nv.NVML_CLOCK_SM)
        rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
        self.samples.append((sm, mx, rs))

    def __enter__(self) -> "ClockSampler":
        import threading

        try:
            import pynvml as nv

            nv.nvmlInit()
            self._nvml = nv
            # NVML enumerates every GPU it can see; map the CUDA ordinal through its UUID.
            import torch

            uuid = getattr(torch.cuda.get_device_properties(self.gpu), "uuid", None)
            try:
                self._handle = nv.nvmlDeviceGetHandleByUUID(f"GPU-{uuid}") if uuid else None
            except Exception:
                self._handle = None
            if self._handle is None:
                self._handle = nv.nvmlDeviceGetHandleByIndex(self.gpu)
            self._sample()
        except Exception:
            self._nvml = None
            return self
        self._stop = threading.Event()

        def loop() -> None:
            while not self._stop.is_set():
                try:
                    self._sample()
                except Exception:
                    return
                self._stop.wait(self.period)

        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc) -> None:
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
            try:
                self._sample()
            except Exception:
                pass
        if self._nvml is not None:
            try:
                self._nvml.nvmlShutdown()
            except Exception:
                pass

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        reasons: set[str] = set()
        nv = self._nvml
        for _, _, rs in self.samples:
            for name, const in self.REASONS.items():
                bit = getattr(nv, const, 0) if nv is not None else 0
                if bit and rs & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[0] for s in self.samples),
                "sm_max_mhz": max(s[1] for s in self.samples), "reasons": sorted(reasons),
                "samples": len(self.samples), "source": "nvml"}


def dist_setup(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    from qwen_image_shardedit_mlx_b200.sharding import max_over_ranks as reduce_max

    return reduce_max(value, device="cuda")


# ----------------------------------------------------------------- our arm


def make_weights(seed: int, device):
    import torch

    from qwen_image_shardedit_mlx_b200.quantize import random_q6

    g = torch.Generator(device=device).manual_seed(seed)
    w1 = random_q6(HIDDEN, DIM, group_size=GROUP, generator=g, device=device)
    w2 = random_q6(DIM, HIDDEN, group_size=GROUP, generator=g, device=device)
    b1 = (torch.randn(HIDDEN, generator=g, device=device) * 0.01).to(torch.bfloat16)
    b2 = (torch.randn(DIM, generator=g, device=device) * 0.01).to(torch.bfloat16)
    return (*w1, b1), (*w2, b2)


def workload_config(world: int) -> dict:
    """The workload both arms run (the reference arm on one host, world 1)."""

    return {
        "workload": WORKLOAD,
        "tokens_per_gpu": TOKENS,
        "dim": DIM,
        "hidden": HIDDEN,
        "group_size": GROUP,
        "global_batch_tokens": TOKENS * world,
        "parallelism": f"token-sharded x{world}, weights replicated, no data-path collective",
        "l2": "no flush: per-step working set ~190 MB (x 21 MB, codes+scales 61 MB, hidden 85 MB, y 21 MB) > 126 MB L2",
    }


def run_ours(args, world: int, rank: int, local: int) -> dict | None:
    import torch

    from qwen_image_shardedit_mlx_b200 import _lib, ops

    dev = torch.device("cuda", local)
    peaks = measured_peaks()
    fc1, fc2 = make_weights(1234, dev)
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    x = torch.randn((TOKENS, DIM), generator=g, device=dev).to(torch.bfloat16)
    hidden = torch.empty((TOKENS, HIDDEN), dtype=torch.bfloat16, device=dev)
    y = torch.empty((TOKENS, DIM), dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)

    # Per-linear launches so each kernel can be timed on the launching stream.
    def fc1_launch():
        ops.q6_linear(x, fc1[0], fc1[1], fc1[2], fc1[3], group_size=GROUP, apply_gelu=True, out=hidden)

    def fc2_launch():
        ops.q6_linear(hidden, fc2[0], fc2[1], fc2[2], fc2[3], group_size=GROUP, out=y)

    for _ in range(max(args.warmup, 3)):
        fc1_launch()
        fc2_launch()
    torch.cuda.synchronize()

    steps = args.steps
    # Timed region: K steps back to back (each kernel may overlap its
    # predecessor's tail through programmatic dependent launch), one event
    # before and one after.
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for i in range(steps):
            fc1_launch()
            fc2_launch()
        end.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    local_ms = start.elapsed_time(end)
    total_ms = max_over_ranks(local_ms, world)
    # Per-kernel durations for the roofline: a second pass of K steps with an
    # event between every pair of launches (which also stops the overlap of
    # one kernel's start with the previous one's tail).
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    for i in range(steps):
        ev[i][0].record(stream)
        fc1_launch()
        ev[i][1].record(stream)
        fc2_launch()
        ev[i][2].record(stream)
    torch.cuda.synchronize()
    fc1_ms = statistics.mean(ev[i][0].elapsed_time(ev[i][1]) for i in range(steps))
    fc2_ms = statistics.mean(ev[i][1].elapsed_time(ev[i][2]) for i in range(steps))
    assert ops.device_error() == 0, "device error word raised during the benchmark"

    # ---- end to end through the public API, host buffers, copies inside the timed region
    from qwen_image_shardedit_mlx_b200 import QuantizedLinear, QwenFeedForward

    ff = QwenFeedForward(QuantizedLinear(*fc1[:3], fc1[3], group_size=GROUP),
                         QuantizedLinear(*fc2[:3], fc2[3], group_size=GROUP))
    # four distinct pinned host batches in, four pinned host outputs, cycled
    xs_host = [x.cpu().pin_memory()] + [
        torch.randn((TOKENS, DIM), generator=torch.Generator().manual_seed(99 + i)).to(torch.bfloat16).pin_memory()
        for i in range(3)]
    ys_host = [torch.empty((TOKENS, DIM), dtype=torch.bfloat16).pin_memory() for _ in range(4)]
    e2e_steps = max(3, min(steps, 20))
    xs = [xs_host[i % 4] for i in range(e2e_steps)]
    ys = [ys_host[i % 4] for i in range(e2e_steps)]
    # (a) the streamed host-buffer API: uploads and downloads overlap the kernels
    # (one untimed pass over the batches first: the first pass over the pinned
    # host buffers runs slower)
    ff.forward_host_stream(xs, ys)
    torch.cuda.synchronize()
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    ff.forward_host_stream(xs, ys)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    # (b) one call at a time: copy in, ff(x), copy out, serially on one stream
    x_dev = torch.empty_like(x)
    barrier(world)
    e0.record(stream)
    for i in range(e2e_steps):
        x_dev.copy_(xs[i], non_blocking=True)
        ys[i].copy_(ff(x_dev), non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_serial_ms = max_over_ranks(e0.elapsed_time(e1), world)
    # (c) the module called on host tensors, one call at a time: each call cuts its rows into
    # chunks whose copies overlap the kernels and returns with the result on the host
    ff.forward_host(xs[0], out=ys[0])
    barrier(world)
    e0.record(stream)
    for i in range(e2e_steps):
        ff.forward_host(xs[i], out=ys[i])
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_call_ms = max_over_ranks(e0.elapsed_time(e1), world)

    # ---- one full MMDiT block (3456 image + 256 text tokens), tensor-parallel over the ranks
    block = None if args.no_block else measure_block(dev, world, rank, form=args.block_form)
    # ---- config 5: the 60-block stack, 8 steps, batch 2, tensor-parallel over the ranks
    stack = None if args.no_stack else measure_stack(dev, world, rank,
                                                     form=block_form(args.block_form, world, STACK_BATCH))

    # ---- skinny-M GEMV side measurement (HBM-bound): a single-GPU figure, taken at N = 1 only
    gemv = None
    if world == 1 and not args.no_gemv:
        gemv = measure_gemv(dev, peaks)

    # ---- the block's memory-bound kernels alone: single-GPU, N = 1 only
    kernels = None
    if world == 1 and not args.no_gemv:
        kernels = measure_kernels(dev, peaks)

    # ---- config 1 and the shape / M / group-size sweep with the LoRA comparison: single-GPU, N = 1 only
    sweep = None
    if world == 1 and not args.no_sweep:
        sweep = measure_sweep(dev, peaks)

    if rank != 0:
        return None
    value = FLOP_PER_STEP * steps * world / (total_ms * 1e-3) / 1e12
    dominant = ("fc2", fc2_ms) if fc2_ms >= fc1_ms else ("fc1", fc1_ms)
    achieved = (FLOP_PER_STEP / 2) / (dominant[1] * 1e-3) / 1e12
    traffic = profiled_traffic().get(dominant[0])
    clock = clocks.summary()
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms / steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights quantised to MLX affine q6 gs64)",
        "config": workload_config(world),
        "fc1_ms": round(fc1_ms, 4),
        "fc2_ms": round(fc2_ms, 4),
        "pct_of_bf16_peak": round(100.0 * value / world / peaks["bf16_tflops"], 2),
        "roofline": {
            "bound": "tensor",
            "kernel": f"q6_linear_tc ({dominant[0]}, 2*3456*3072*12288 FLOP per launch)",
            "achieved": round(achieved, 2),
            "peak": peaks["bf16_tflops"],
            "unit": "TFLOP/s",
            "frac": round(achieved / peaks["bf16_tflops"], 4),
            "peak_source": f"{peaks['source']} (burst cuBLAS bf16)",
            "traffic": traffic,
        },
        "e2e": {
            "value": round(FLOP_PER_STEP * e2e_steps * world / (e2e_ms * 1e-3) / 1e12, 2),
            "unit": "TFLOP/s",
            "h2d_bytes_per_step": TOKENS * DIM * 2,
            "d2h_bytes_per_step": TOKENS * DIM * 2,
            "api": "QwenFeedForward.forward_host_stream: pinned host batches in and out, uploads and downloads overlapping the kernels",
            "serial_value": round(FLOP_PER_STEP * e2e_steps * world / (e2e_serial_ms * 1e-3) / 1e12, 2),
            "serial_api": "QwenFeedForward(x) one call at a time: copy in, ff, copy out on one stream",
            "host_call_value": round(FLOP_PER_STEP * e2e_steps * world / (e2e_call_ms * 1e-3) / 1e12, 2),
            "host_call_api": "QwenFeedForward(x_host) one call at a time on a pinned host tensor: 4 chunks of 864 "
                             "rows, each chunk's upload / download overlapping the other chunks' kernels; "
                             "returns with the result on the host",
        },
        "gpu_launches": 2 * steps,
        "kernel_timing": "fc1_ms / fc2_ms and roofline.achieved from a second pass of the same steps with an event "
                         "between launches; value from the timed pass without them",
        "token_tile": int(_lib.lib().q6_tensor_token_tile(TOKENS, HIDDEN)),
        "clocks": clock,
    }
    if gemv is not None:
        line["gemv"] = gemv
    if kernels is not None:
        line["kernels"] = kernels
    if sweep is not None:
        line["c1"] = sweep.pop("c1")
        line["sweep"] = sweep
    if block is not None:
        line["block"] = block
    if stack is not None:
        line["stack"] = stack
    if world == 1 and not args.no_cpu_baseline:  # the host-core baseline is taken at N = 1 only
        line["cpu_baseline"] = cpu_baseline_port()
    return line


BLOCK_IMG, BLOCK_TXT, BLOCK_HEADS = 3456, 256, 24
STACK_BLOCKS, STACK_STEPS, STACK_BATCH = 60, 8, 2


def _graph_ms(run, world: int, steps: int) -> tuple[float, float]:
    """(graph-replay ms, eager ms) per call of ``run``: device time from CUDA
    events over ``steps`` calls, max over ranks.  The graph holds the whole
    call (every launch and collective), captured once after a warm-up."""

    import torch

    stream = torch.cuda.current_stream()
    for _ in range(3):
        run()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)

    def timed(fn) -> float:
        barrier(world)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        return max_over_ranks(e0.elapsed_time(e1) / steps, world)

    eager_ms = timed(run)
    side = torch.cuda.Stream()
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        run()
    stream.wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run()
    graph.replay()
    torch.cuda.synchronize()
    ms = timed(graph.replay)
    del graph  # holds NCCL work on N > 1: released before the process group goes
    torch.cuda.synchronize()
    return ms, eager_ms


def _block_inputs(dev, batch: int, seed: int):
    import torch

    from qwen_image_shardedit_mlx_b200.block import joint_rope, qwen_rope_angles, rope_tables

    g = torch.Generator(device=dev).manual_seed(seed)
    seq = BLOCK_IMG + BLOCK_TXT
    x = torch.randn((batch * seq, DIM), generator=g, device=dev).to(torch.bfloat16)
    temb = torch.randn((batch, DIM), generator=g, device=dev).to(torch.bfloat16)
    ia, ta = qwen_rope_angles([(36, 48), (36, 48)], BLOCK_TXT)
    return x, temb, joint_rope(rope_tables(ia, ta, dev)), seq


BLOCK_FORMS = {
    "cp": "context-parallel: every rank the full weights; a batch's samples first split over rank groups "
          "(gcd(N, batch) groups, e.g. one sample of the CFG pair per half of the GPUs), then each sample's joint "
          "rows split over its group's ranks through the whole block, keys and values all-gathered (NCCL) within "
          "the group for the attention",
    "tp-peer": "tensor-parallel heads and FF columns with sequence-parallel rows between the GEMMs; fused "
               "peer-memory reduce + residual + adaLN + gather kernels and 4 barriers per block",
    "tp-nccl": "tensor-parallel heads and FF columns with sequence-parallel rows between the GEMMs; 2 all-gathers "
               "+ 2 reduce-scatters (NCCL) per block",
}


def block_form(choice: str, world: int, batch: int) -> str:
    """The multi-GPU block form for ``--block-form``: ``auto`` takes the form
    measured faster on B200.  A batch that splits over the GPUs (the CFG
    pair on an even count) runs context-parallel with one sample per group of
    ranks (no communication at 2 GPUs).  One sample runs tensor-parallel with
    peer-memory collectives at 2 GPUs (block 0.679 ms against cp's 0.718 ms)
    and context-parallel from 4, where the tensor-parallel GEMMs shrink to
    K = 384 and 1152 columns (8 GPUs: 0.579 ms against cp's 0.408 ms)."""

    if choice != "auto":
        return choice
    import math

    if batch > 1 and math.gcd(world, batch) > 1:
        return "cp"
    return "tp-peer" if world <= 2 else "cp"


def _block_runner(form: str, full, world: int, rank: int, x, temb, rope_j, batch: int, seq: int):
    """A per-rank forward of one multi-GPU block form over this rank's rows of x."""

    from qwen_image_shardedit_mlx_b200.block import ContextParallelQwenBlock, TensorParallelQwenBlock, sample_groups

    if form == "cp":
        samples, size, r_in, grp = sample_groups(world, rank, batch)
        nb = samples.stop - samples.start
        blk = ContextParallelQwenBlock(full, size, r_in, group=grp)
        x_local = blk.local_rows(x.view(batch, seq, -1)[samples].reshape(nb * seq, -1), nb, seq)
        t = temb[samples]
        return lambda: blk.forward_local(x_local, t, rope_j, nb, seq, BLOCK_TXT)
    blk = TensorParallelQwenBlock(full, world, rank, comm=form[3:])
    rows_local = x.shape[0] // world
    x_local = x[rank * rows_local:(rank + 1) * rows_local].contiguous()
    return lambda: blk.finish(blk.forward_local(x_local, temb, rope_j, batch, seq, BLOCK_TXT))


def measure_block(dev, world: int, rank: int, steps: int = 10, form: str = "auto") -> dict | None:
    """Device time of one Qwen-Image MMDiT block forward (3456 image + 256
    text tokens, all 14 linears q6 gs64, joint attention over 3712 tokens), at
    batch 1 (config 3) and batch 2 (the per-block cost of config 5's CFG pair).
    With N ranks every multi-GPU form is timed in the same run (``forms_ms``)
    and ``ms`` is the one ``form`` names (BLOCK_FORMS); rank 0 also times the
    single-GPU block, so the line carries the strong-scaling efficiency
    ms_1gpu / (N ms)."""

    import torch

    from qwen_image_shardedit_mlx_b200 import ops
    from qwen_image_shardedit_mlx_b200.block import QwenTransformerBlock, TensorParallelQwenBlock, block_flops

    g = torch.Generator(device=dev).manual_seed(2025)  # the same block on every rank
    full = QwenTransformerBlock.random(DIM, BLOCK_HEADS, generator=g, device=dev)
    out = {}
    choice = form
    for batch in (1, 2):
        form = block_form(choice, world, batch)
        x, temb, rope_j, seq = _block_inputs(dev, batch, 7 + batch)
        y = torch.empty_like(x)
        one = lambda: full.forward_joint(x, temb, rope_j, batch, BLOCK_TXT, out=y)  # noqa: E731
        ms_tp1 = ms_one_stream = None
        forms_ms = None
        if world == 1:
            ms, eager_ms = _graph_ms(one, world, steps)
            ms_1 = ms
            # both streams' GEMMs in order on one CUDA stream (no fork / join)
            full.overlap_streams = False
            ms_one_stream, _ = _graph_ms(one, 1, steps)
            full.overlap_streams = True
            # the tensor-parallel form on one rank: the cost of its structure alone
            tp1 = TensorParallelQwenBlock(full, 1, 0, comm="peer")
            ms_tp1, _ = _graph_ms(lambda: tp1.finish(tp1.forward_local(x, temb, rope_j, batch, seq, BLOCK_TXT)),
                                  1, steps)
            del tp1
        else:
            forms_ms = {}
            eager_ms = None
            for f in BLOCK_FORMS:  # every rank takes the same forms in the same order
                run = _block_runner(f, full, world, rank, x, temb, rope_j, batch, seq)
                f_ms, f_eager = _graph_ms(run, world, steps)
                forms_ms[f] = round(f_ms, 4)
                if f == form:
                    ms, eager_ms = f_ms, f_eager
                del run
                torch.cuda.empty_cache()
            ms_1 = None
            if rank == 0:
                ms_1, _ = _graph_ms(one, 1, steps)
            barrier(world)
        torch.cuda.synchronize()
        assert ops.device_error() == 0, "block benchmark raised the device error word"
        flop = batch * block_flops(BLOCK_IMG, BLOCK_TXT, DIM)
        out[f"b{batch}"] = {
            "ms": round(ms, 4), "TFLOP/s": round(flop / (ms * 1e-3) / 1e12, 1), "eager_ms": round(eager_ms, 4),
            "ms_1gpu": None if ms_1 is None else round(ms_1, 4),
            "form": form if world > 1 else None,
            "forms_ms": forms_ms,
            "ms_tp_form_1gpu": None if ms_tp1 is None else round(ms_tp1, 4),
            "ms_one_stream_1gpu": None if ms_one_stream is None else round(ms_one_stream, 4),
            "efficiency_vs_1gpu": None if ms_1 is None else round(ms_1 / (world * ms), 4),
            "batch": batch, "flop_per_call": flop,
        }
    if rank != 0:
        return None
    res = dict(out["b1"])
    res.update({
        "n_gpus": world,
        "batch2": out["b2"],
        "parallelism": "single GPU" if world == 1 else
        f"batch 1: {BLOCK_FORMS[out['b1']['form']]}; batch 2: {BLOCK_FORMS[out['b2']['form']]} "
        f"(x{world}; forms_ms: every form, same run)",
        "shape": f"{BLOCK_IMG} image + {BLOCK_TXT} text tokens, hidden {DIM}, {BLOCK_HEADS} heads x 128, "
                 "FF 4x, all 14 linears q6 gs64",
        "steps": steps,
        "note": "device time per block forward replayed from a CUDA graph (eager_ms: launched from Python each "
                "time); CUDA events, max over ranks; attention is the library scaled_dot_product_attention kernel; "
                "ms_1gpu is the same block on one GPU timed on rank 0 in the same run; ms_tp_form_1gpu (one GPU "
                "only) is the tensor-parallel form run on a single rank, the cost of its layout and kernels alone; "
                "ms_one_stream_1gpu runs the text- and image-stream GEMMs in order on one CUDA stream instead of "
                "overlapping them on two",
    })
    return res


def measure_stack(dev, world: int, rank: int, blocks: int = STACK_BLOCKS, steps: int = STACK_STEPS,
                  form: str = "cp") -> dict | None:
    """Config 5: the 60-block q6 MMDiT stack, batch 2 (CFG cond / uncond),
    3456 image + 256 text tokens per sample, 8 denoising steps, over the
    ranks in the multi-GPU ``form`` (BLOCK_FORMS).  Each rank builds 60 random
    blocks (seeded per block; the full weights for the context-parallel form,
    its shards for the tensor-parallel ones) and keeps its rows sharded from
    block to block (the tensor-parallel forms fold each block's residual add
    into the next block's first modulate; on one GPU that form runs).  Every
    block's modulation vectors come first, 1 / N of the GEMVs per rank and one
    all-gather.  One denoising step (every block, a new timestep embedding) is
    captured in a CUDA graph and replayed ``steps`` times; the time is device
    time, max over ranks.  Only the block stack is timed (the model's input
    and output projections and the sampler are outside the q6 path)."""

    import torch

    from qwen_image_shardedit_mlx_b200 import ops
    from qwen_image_shardedit_mlx_b200.block import (ContextParallelQwenBlock, QwenTransformerBlock,
                                                     TensorParallelQwenBlock, block_flops, sample_groups,
                                                     stack_modulations)

    cp = form == "cp" and world > 1
    batch = STACK_BATCH
    samples, size, r_in, grp = sample_groups(world, rank, batch) if cp else (slice(0, batch), world, rank, None)
    nb = samples.stop - samples.start
    stack = []
    for i in range(blocks):
        g = torch.Generator(device=dev).manual_seed(10_000 + i)
        full = QwenTransformerBlock.random(DIM, BLOCK_HEADS, generator=g, device=dev)
        if cp:
            stack.append(ContextParallelQwenBlock(full, size, r_in, group=grp))
        else:
            stack.append(TensorParallelQwenBlock(full, world, rank, comm=form[3:] if world > 1 else "nccl"))
        del full
    torch.cuda.empty_cache()
    x, _, rope_j, seq = _block_inputs(dev, batch, 99)
    if cp:
        x_local = stack[0].local_rows(x.view(batch, seq, -1)[samples].reshape(nb * seq, -1), nb, seq)
    else:
        rows_local = x.shape[0] // world
        x_local = x[rank * rows_local:(rank + 1) * rows_local].contiguous()
    g = torch.Generator(device=dev).manual_seed(5)
    tembs = [torch.randn((batch, DIM), generator=g, device=dev).to(torch.bfloat16) for _ in range(steps)]
    temb = tembs[0].clone()

    def one_step():
        if cp:
            # this group's samples: every block's modulation vectors first, the GEMVs split
            # over the group's ranks and one all-gather
            t = temb[samples]
            mods = stack_modulations(stack, t, size, r_in, group=grp)
            y = x_local
            for i, blk in enumerate(stack):
                y = blk.forward_local(y, t, rope_j, nb, seq, BLOCK_TXT, mod=mods[i])
            return y
        # every block's modulation vectors first, 1 / N of the GEMVs per rank and one all-gather
        mods = stack_modulations(stack, temb, world, rank)
        pending = stack[0].forward_local(x_local, temb, rope_j, batch, seq, BLOCK_TXT, mod=mods[0])
        for i, blk in enumerate(stack[1:], start=1):
            pending = blk.forward_local_pending(pending, temb, rope_j, batch, seq, BLOCK_TXT, mod=mods[i])
        return stack[-1].finish(pending)

    stream = torch.cuda.current_stream()
    one_step()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        one_step()
    stream.wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y = one_step()
    for i in range(2):  # warm-up replays
        temb.copy_(tembs[i % steps])
        graph.replay()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(steps):
        temb.copy_(tembs[i])  # the step's timestep embedding (3 KB device copy, part of the step)
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    total_ms = max_over_ranks(e0.elapsed_time(e1), world)
    finite = bool(torch.isfinite(y).all())
    del graph
    torch.cuda.synchronize()
    assert ops.device_error() == 0 and finite, "stack benchmark raised the device error word or non-finite output"
    del stack
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    flop = steps * blocks * batch * block_flops(BLOCK_IMG, BLOCK_TXT, DIM)
    return {
        "ms_per_step": round(total_ms / steps, 3), "total_ms": round(total_ms, 2), "steps": steps, "blocks": blocks,
        "batch": batch, "n_gpus": world, "TFLOP/s": round(flop / (total_ms * 1e-3) / 1e12, 1),
        "parallelism": "single GPU" if world == 1 else f"{BLOCK_FORMS[form]} (x{world})",
        "form": form if world > 1 else None,
        "shape": f"{blocks} blocks x batch {batch} x ({BLOCK_IMG} image + {BLOCK_TXT} text tokens), hidden {DIM}, "
                 "all linears q6 gs64",
        "note": "one denoising step (all blocks) captured in a CUDA graph and replayed per step with that step's "
                "timestep embedding; device time, max over ranks; block stack only",
    }


GEMV_CASES = [
    # (name, N, K, M): the few-row shapes of the block (q6_linear_profile.py:144-159)
    ("m1", 12288, 3072, 1),          # 3072 -> 12288 at one token row
    ("m2", 12288, 3072, 2),          # two rows (a CFG pair)
    ("m16", 12288, 3072, 16),        # the skinny-M target shape
    ("m1_k12288", 3072, 12288, 1),   # fc2-shaped (12288 -> 3072) at one row
    ("mod_m2", 18432, 3072, 2),      # the adaLN modulation linear at batch 2
]


def measure_gemv(dev, peaks, only: str | None = None) -> dict:
    """q6 linears for a few token rows (GEMV_CASES), rotating weight copies
    whose total exceeds L2 four times so every launch streams its weights from
    HBM; device time per launch from a CUDA graph of back-to-back launches,
    reported as HBM GB/s of the algorithmic bytes (codes, scales, biases, x, y)."""

    import torch

    from qwen_image_shardedit_mlx_b200 import ops
    from qwen_image_shardedit_mlx_b200.quantize import random_q6

    g = torch.Generator(device=dev).manual_seed(77)
    out = {}
    shapes: dict[tuple[int, int], list] = {}
    wanted = None if not only else set(only.split(","))
    unknown = (wanted or set()) - {c[0] for c in GEMV_CASES}
    if unknown:
        raise ValueError(f"unknown GEMV case(s) {sorted(unknown)}")
    for name, n, k, m in GEMV_CASES:
        if wanted is not None and name not in wanted:
            continue
        shapes.setdefault((n, k), []).append((name, m))
    for (n, k), cases in shapes.items():
        per_copy = n * k * 6 // 8 + 2 * 2 * n * (k // GROUP)
        count = max(8, int(4 * L2_BYTES // per_copy) + 1)
        w0 = random_q6(n, k, group_size=GROUP, generator=g, device=dev)
        copies = [w0] + [tuple(t.clone() for t in w0) for _ in range(count - 1)]
        for name, m in cases:
            x = torch.randn((m, k), generator=g, device=dev).to(torch.bfloat16)
            y = torch.empty((m, n), dtype=torch.bfloat16, device=dev)

            def launch(i, x=x, y=y):
                w, s, b = copies[i % count]
                ops.q6_linear(x, w, s, b, group_size=GROUP, out=y)

            us = _time_launches(launch, count, reps=8)
            nbytes = per_copy + 2 * m * (k + n)
            gbs = nbytes / (us * 1e-6) / 1e9
            out[name] = {"n": n, "k": k, "m": m, "us": round(us, 2), "GB/s": round(gbs, 1),
                         "frac_hbm": round(gbs / peaks["hbm_gbs"], 4), "path": ops.last_path(), "bytes": nbytes}
        del copies, w0
        torch.cuda.empty_cache()
    out["note"] = ("gs64; weight copies rotating over > 4x L2 per shape, one CUDA graph of back-to-back launches, "
                   "device time; frac_hbm against the measured copy bandwidth")
    return out


def measure_kernels(dev, peaks) -> dict:
    """The block's memory-bound kernels alone at the block's shapes (3712
    joint rows of 3072, 24 heads): the residual add + adaLN modulate, the
    QK-RMSNorm + RoPE (in place on the q columns of a qkv buffer) and the LoRA
    pre-pass x @ A (3456 x 3072 by rank 64).  Inputs rotate over copies
    totalling more than L2 so every launch reads HBM; device time per launch
    from a CUDA graph of back-to-back launches, reported as GB/s of the
    algorithmic bytes (each element read and written once)."""

    import torch

    from qwen_image_shardedit_mlx_b200 import ops
    from qwen_image_shardedit_mlx_b200.block import (ModulationVectors, add_layernorm_modulate,
                                                     qk_rmsnorm_rope_joint_, qwen_rope_angles, rope_tables,
                                                     joint_rope)

    g = torch.Generator(device=dev).manual_seed(31)
    rows, seq = BLOCK_IMG + BLOCK_TXT, BLOCK_IMG + BLOCK_TXT
    out = {}

    def rate(name, us, nbytes, **extra):
        gbs = nbytes / (us * 1e-6) / 1e9
        out[name] = {"us": round(us, 2), "GB/s": round(gbs, 1), "frac_hbm": round(gbs / peaks["hbm_gbs"], 4),
                     "bytes": nbytes, **extra}

    # residual add + adaLN modulate: x + add read, h and y written
    copies = 3
    xs = [torch.randn((rows, DIM), generator=g, device=dev).to(torch.bfloat16) for _ in range(copies)]
    adds = [torch.randn((rows, DIM), generator=g, device=dev).to(torch.bfloat16) for _ in range(copies)]
    hs = [torch.empty_like(xs[0]) for _ in range(copies)]
    ys = [torch.empty_like(xs[0]) for _ in range(copies)]
    vec = ModulationVectors(torch.randn((1, 2, 6, DIM), generator=g, device=dev).to(torch.bfloat16))
    us = _time_launches(lambda i: add_layernorm_modulate(xs[i % copies], vec.shift2, vec.scale2, add=adds[i % copies],
                                                         h_out=hs[i % copies], out=ys[i % copies], seq_len=seq,
                                                         text_len=BLOCK_TXT), copies)
    rate("add_layernorm_modulate", us, 4 * rows * DIM * 2, rows=rows, dim=DIM)
    us = _time_launches(lambda i: add_layernorm_modulate(xs[i % copies], vec.shift1, vec.scale1, out=ys[i % copies],
                                                         seq_len=seq, text_len=BLOCK_TXT), copies)
    rate("layernorm_modulate", us, 2 * rows * DIM * 2, rows=rows, dim=DIM)
    del xs, adds, hs, ys
    # QK-RMSNorm + RoPE on the q columns of a [rows, 3 D] qkv buffer
    qkvs = [torch.randn((rows, 3 * DIM), generator=g, device=dev).to(torch.bfloat16) for _ in range(copies)]
    ia, ta = qwen_rope_angles([(36, 48), (36, 48)], BLOCK_TXT)
    cos, sin = joint_rope(rope_tables(ia, ta, dev))
    wq = (1.0 + 0.1 * torch.randn((128,), generator=g, device=dev)).to(torch.bfloat16)
    us = _time_launches(lambda i: qk_rmsnorm_rope_joint_(qkvs[i % copies][:, :DIM], wq, wq, cos, sin, seq_len=seq,
                                                         text_len=BLOCK_TXT), copies)
    rate("qk_rmsnorm_rope", us, 2 * rows * DIM * 2, rows=rows, heads=BLOCK_HEADS)
    del qkvs
    # LoRA pre-pass: x read once, xa written
    xs = [torch.randn((TOKENS, DIM), generator=g, device=dev).to(torch.bfloat16) for _ in range(4)]
    a = (torch.randn((DIM, 64), generator=g, device=dev) * 0.01).to(torch.bfloat16)
    xa = torch.empty((TOKENS, 64), dtype=torch.bfloat16, device=dev)
    us = _time_launches(lambda i: ops.lora_xa(xs[i % 4], a, out=xa), 4)
    rate("lora_xa_rank64", us, TOKENS * DIM * 2 + DIM * 64 * 2 + TOKENS * 64 * 2, rows=TOKENS, rank=64)
    del xs
    torch.cuda.empty_cache()
    assert ops.device_error() == 0, "kernel benchmark raised the device error word"
    out["note"] = ("device time per launch in a CUDA graph of back-to-back launches over input copies larger than "
                   "L2; GB/s of the algorithmic bytes against the measured copy bandwidth")
    return out


SWEEP_SHAPES = [(3072, 3072), (12288, 3072), (3072, 12288), (18432, 3072)]  # (N, K): q6_linear_profile.py:144-159
SWEEP_M = (1, 16, 128, 512, 1728, 3456, 8192)
SWEEP_GS = (32, 64, 128)


def _time_launches(launch, count: int, reps: int = 5) -> float:
    """Mean device microseconds per launch of ``launch(i)`` for i in 0..count-1,
    replayed from a CUDA graph of back-to-back launches (no host cost)."""

    import torch

    for i in range(count):
        launch(i)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for i in range(count):
            launch(i)
    torch.cuda.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    del graph
    return e0.elapsed_time(e1) * 1e3 / (reps * count)


def measure_sweep(dev, peaks) -> dict:
    """Config 1 (x [1728, 3072] -> 12288, gs64) and the config-4 grid: the
    block's four projection shapes x M in {1, 16, 128, 512, 1728, 3456, 8192}
    x group sizes {32, 64, 128}, no bias (benchmarks/benchmark_qwen_gemm.py:119-200
    times the same grid).  Each point is timed from a CUDA graph of
    back-to-back launches; below 512 tokens the launches rotate over weight
    copies whose total exceeds L2 four times, so the weights stream from HBM.
    A point is HBM-bound when its FLOP per algorithmic byte is below the
    measured ridge (bf16 peak / HBM bandwidth), else tensor-bound; ``frac`` is
    against that roofline.  Plus rank-64 LoRA at config 1 and image-FF fc1:
    plain q6, unfused (pre-pass, q6, then a separate s (xa @ B) GEMM added to
    y) and fused into the q6 tile."""

    import torch

    from qwen_image_shardedit_mlx_b200 import ops
    from qwen_image_shardedit_mlx_b200.quantize import random_q6

    g = torch.Generator(device=dev).manual_seed(4096)
    ridge = peaks["bf16_tflops"] * 1e12 / (peaks["hbm_gbs"] * 1e9)
    xs = {m: torch.randn((m, 12288), generator=g, device=dev).to(torch.bfloat16) for m in SWEEP_M}
    points = []
    for (n, k) in SWEEP_SHAPES:
        for gs in SWEEP_GS:
            w0 = random_q6(n, k, group_size=gs, generator=g, device=dev)
            per_copy = n * k * 6 // 8 + 2 * 2 * n * (k // gs)
            count = max(2, -(-4 * L2_BYTES // per_copy))
            copies = [w0] + [tuple(t.clone() for t in w0) for _ in range(count - 1)]
            for m in SWEEP_M:
                x = xs[m][:, :k].contiguous()
                y = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
                rot = count if m < 512 else 1

                def launch(i, x=x, y=y, gs=gs, rot=rot):
                    w, s, b = copies[i % rot]
                    ops.q6_linear(x, w, s, b, group_size=gs, out=y)

                us = _time_launches(launch, max(rot, 8) if m < 512 else 8)
                flop = 2.0 * m * n * k
                nbytes = per_copy + 2 * m * (k + n)
                bound = "hbm" if flop / nbytes < ridge else "tensor"
                tflops = flop / (us * 1e-6) / 1e12
                gbs = nbytes / (us * 1e-6) / 1e9
                frac = gbs / peaks["hbm_gbs"] if bound == "hbm" else tflops / peaks["bf16_tflops"]
                points.append({"n": n, "k": k, "m": m, "gs": gs, "us": round(us, 2), "TFLOP/s": round(tflops, 2),
                               "GB/s": round(gbs, 1), "bound": bound, "frac": round(frac, 4),
                               "path": ops.last_path()})
            del copies, w0
            torch.cuda.empty_cache()

    c1 = next(p for p in points if (p["n"], p["k"], p["m"], p["gs"]) == (12288, 3072, 1728, 64))

    # rank-64 LoRA: plain vs unfused vs fused
    lora = {}
    for name, (m, n, k, gelu) in {"config1": (1728, 12288, 3072, False), "image_ff_fc1": (3456, 12288, 3072, True)}.items():
        w, s, b = random_q6(n, k, group_size=64, generator=g, device=dev)
        bias = (torch.randn(n, generator=g, device=dev) * 0.01).to(torch.bfloat16)
        a_l = (torch.randn((k, 64), generator=g, device=dev) * 0.01).to(torch.bfloat16)
        b_l = (torch.randn((64, n), generator=g, device=dev) * 0.01).to(torch.bfloat16)
        x = xs[m][:, :k].contiguous()
        y = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
        xa = torch.empty((m, 64), dtype=torch.bfloat16, device=dev)

        def plain(i, x=x, w=w, s=s, b=b, bias=bias, y=y, gelu=gelu):
            ops.q6_linear(x, w, s, b, bias, group_size=64, apply_gelu=gelu, out=y)

        def unfused(i, x=x, w=w, s=s, b=b, bias=bias, y=y, gelu=gelu, a_l=a_l, b_l=b_l, xa=xa):
            # the reference's order: y = act(q6(x) + bias + s (x A) B) needs the delta before the
            # activation, so without fusion the q6 GEMM runs without its epilogue activation
            ops.lora_xa(x, a_l, out=xa)
            ops.q6_linear(x, w, s, b, group_size=64, out=y)
            y.addmm_(xa, b_l, alpha=1.0)
            if gelu:
                y.copy_(torch.nn.functional.gelu(y + bias, approximate="tanh"))
            else:
                y.add_(bias)

        b_t = b_l.t().contiguous()  # what QuantizedLinear.set_lora keeps beside B: [N, r]

        def fused(i, x=x, w=w, s=s, b=b, bias=bias, y=y, gelu=gelu, a_l=a_l, b_l=b_l, b_t=b_t):
            ops.q6_linear(x, w, s, b, bias, group_size=64, apply_gelu=gelu, lora=(a_l, b_l, 1.0), lora_b_nmajor=b_t,
                          out=y)

        t_plain = _time_launches(plain, 8)
        t_unf = _time_launches(unfused, 8)
        t_fused = _time_launches(fused, 8)
        lora[name] = {"m": m, "n": n, "k": k, "rank": 64, "gelu": gelu, "plain_us": round(t_plain, 2),
                      "unfused_us": round(t_unf, 2), "fused_us": round(t_fused, 2),
                      "fused_overhead_pct": round(100.0 * (t_fused / t_plain - 1.0), 2),
                      "unfused_overhead_pct": round(100.0 * (t_unf / t_plain - 1.0), 2)}
    tensor_pts = [p for p in points if p["bound"] == "tensor"]
    hbm_pts = [p for p in points if p["bound"] == "hbm"]
    return {
        "c1": {**c1, "workload": "config 1: x [1728, 3072] bf16 -> q6 gs64 3072->12288, no bias",
               "roofline_peak": peaks["bf16_tflops"]},
        "points": points,
        "lora_rank64": lora,
        "summary": {
            "tensor_points": len(tensor_pts), "hbm_points": len(hbm_pts),
            "tensor_frac_median": round(statistics.median(p["frac"] for p in tensor_pts), 4) if tensor_pts else None,
            "hbm_frac_median": round(statistics.median(p["frac"] for p in hbm_pts), 4) if hbm_pts else None,
            "ridge_flop_per_byte": round(ridge, 1),
        },
        "note": "device time per launch from CUDA graphs of back-to-back launches; weights rotate over copies "
                "totalling > 4x L2 below 512 tokens; no bias; frac against the measured peak of the point's bound",
    }


# ------------------------------------------------------------ host baselines


def cpu_baseline_port(budget_s: float = 12.0) -> dict:
    """The oracle's torch-CPU restatement (dequantise, then matmul) on a token sample."""

    import torch

    from oracle.cpu_port import mlp_port_flops, time_mlp_port

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    tokens, seconds, steps = time_mlp_port(TOKENS, DIM, HIDDEN, GROUP, budget_s=budget_s)
    flops = mlp_port_flops(tokens, DIM, HIDDEN) * steps
    return {"value": round(flops / seconds / 1e12, 4), "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{steps} step(s) of {tokens} tokens through fc1+GELU+fc2 (bf16 weights dequantised once before timing, torch bf16 matmul)"}


def run_reference(args, world: int, rank: int) -> dict | None:
    """The reference's own q6 kernel (SOURCE_QMM_T compiled for the host) on
    full 3456-token steps of the same MLP workload, rank 0 only."""

    if rank != 0:
        return None
    from oracle.cpu_port import time_reference_kernel_mlp

    res = time_reference_kernel_mlp(DIM, HIDDEN, GROUP, tokens=TOKENS, steps=args.steps)
    value = res["tflops"]
    seconds_per_step = FLOP_PER_STEP / (value * 1e12)
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 6),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": res["steps"],
        "warmup": args.warmup,
        "ms_per_step": round(seconds_per_step * 1e3, 1),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights quantised to MLX affine q6 gs64)",
        "config": workload_config(1),
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": res["cores"], "kind": res["kind"],
                         "sample": res["sample"]},
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main() -> int:
    args = parse_args()
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        line = run_reference(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0
    world, rank, local = dist_setup(args)
    try:
        if args.only:
            import torch

            dev = torch.device("cuda", local)
            fn = {"block": lambda: measure_block(dev, world, rank, form=args.block_form),
                  "stack": lambda: measure_stack(dev, world, rank,
                                                 form=block_form(args.block_form, world, STACK_BATCH)),
                  "gemv": lambda: measure_gemv(dev, measured_peaks(), args.gemv_case) if rank == 0 else None,
                  "sweep": lambda: measure_sweep(dev, measured_peaks()) if rank == 0 else None,
                  "kernels": lambda: measure_kernels(dev, measured_peaks()) if rank == 0 else None}[args.only]
            res = fn()
            if rank == 0:
                print(json.dumps({"only": args.only, args.only: res}), flush=True)
            return 0
        line = run_ours(args, world, rank, local)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
