"""Benchmark of the fused AdamW-SR step at the Llama-3-8B shape.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

A step is one optimizer step of the whole parameter set: 291 tensors,
8,030,261,248 BF16 parameters with BF16 gradients ~N(0, 1e-4), FP8 E4M3
stochastic first moment and BF16 stochastic second moment, lr 3e-4, weight
decay 0.1, seed 7.  With N GPUs the step is sharded ZeRO-1 style (each rank
updates its flat shard, states exist only for it) and the updated BF16
parameters are reassembled on every rank inside the timed step: the fused
kernel stores them into the peers' replicas over NVLink (an NCCL all-gather
when peer mappings are unavailable).  Inputs are synthetic and resident in HBM (56 GB per GPU
at N=1, far above the 126 MB L2, so no cache flush is needed).

Prints one JSON line (rank 0): value = parameters updated per second by the
whole job; roofline = the fused kernel's algorithmic HBM bytes per second
against the measured copy bandwidth; e2e = the same step through the public
optimizer API with the gradients copied in from pinned host memory and the
updated parameters copied back every step; cpu_baseline = the CPU oracle on
this host's cores over a bounded sample of the same workload.

Other workloads of the same path (one GPU; not the headline):
    --workload sgdm-gpt2   momentum SGD at the GPT-2-small shape (148 tensors,
                           124,439,808 FP32 params, BF16 stochastic momentum)
    --workload cast        the standalone cast, FP32 -> BF16/FP16/E4M3/E5M2 x
                           {stochastic, nearest}, one line per target and rule
    --workload adamw-70b   AdamW at the Llama-3-70B shape with FP16 stochastic
                           states on 4 or 8 GPUs, everything sharded (see
                           run_adamw_70b)
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

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "stochastic-rounding-pytorch_b200"))

METRIC = "AdamW-SR step params/sec & HBM GB/s (% of peak) at 8B shape, 1/2/4/8 B200"
# Algorithmic bytes per parameter: read p, g, m, v; write p, m, v
# (BF16 p/g = 2 B, E4M3 m = 1 B, BF16 v = 2 B): 2+2+1+2 + 2+1+2 = 12.
BYTES_PER_PARAM = 12
# DRAM bytes per parameter of one AdamW launch measured by ncu
# (dram__bytes_read.sum + dram__bytes_write.sum = 5.197 GB over the 436,228,096
# parameters of the 2-layer profiling case; profiles/adamw_kernel_llama3-8b.md).
# Traffic grows in proportion to the parameters, so a full launch moves this
# many bytes per parameter.
MEASURED_TRAFFIC_PER_PARAM = 11.913
FALLBACK_HBM_GBS = 6650.0


def parse_args(argv=None):
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=10)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=("b200", "reference"), default="b200")
    parser.add_argument("--e2e-steps", type=int, default=3)
    parser.add_argument("--cpu-seconds", type=float, default=12.0,
                        help="CPU work budget of the CPU baseline sample")
    parser.add_argument("--no-e2e", action="store_true")
    parser.add_argument("--layers", type=int, default=32,
                        help="decoder layers of the Llama-3-8B shape (profiling uses fewer)")
    parser.add_argument("--no-embeddings", action="store_true",
                        help="drop the two 128256x4096 matrices (profiling case)")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--workload", choices=("adamw-8b", "sgdm-gpt2", "cast", "adamw-70b"),
                        default="adamw-8b")
    parser.add_argument("--gather", choices=("auto", "fused", "copy", "nccl"), default="auto",
                        help="how the sharded step reassembles the parameters at N>1")
    parser.add_argument("--chunks", type=int, default=32,
                        help="tile chunks of the pipelined exchange (--gather copy)")
    parser.add_argument("--cast-elems", type=int, default=1 << 30,
                        help="elements of the cast workload (FP32 input)")
    return parser.parse_args(argv)


def measured_hbm_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (copy)"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback 6.65 TB/s (MEASURED_PEAKS.json absent)"


# ------------------------------------------------------------ distributed --

def init_distributed(n_gpus):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch with torchrun")
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value, world):
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- clocks --

class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while active."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, index):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - clocks are reported when NVML is usable
            self._nvml = None
        self._thread = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self._nvml.nvmlDeviceGetClockInfo(
                    self._handle, self._nvml.NVML_CLOCK_SM))
                mask = self._nvml.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                self.reasons |= {n for n, bit in self.REASONS.items() if mask & bit}
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(0.1)

    def __enter__(self):
        if self._nvml is not None:
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread.is_alive():
            self._thread.join()

    def report(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


# -------------------------------------------------------------- workload --

def build_workload(world, rank, layers=32, embeddings=True, gather="auto", chunks=32):
    """Flat BF16 parameter and gradient buffers holding the 291 tensors; the
    optimizer (ZeRO-1 when world > 1) over views of them."""
    import torch

    from sr_states import StateFormat
    from sr_states.distributed import ZeroAdamW
    from sr_states.shapes import llama3_8b

    shapes = [s for name, s in llama3_8b()
              if (embeddings or name not in ("embed_tokens", "lm_head"))
              and not (name.startswith("layers.") and int(name.split(".")[1]) >= layers)]
    total = sum(math.prod(s) for s in shapes)
    device = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=device).manual_seed(7)
    flat_p = torch.empty(total, dtype=torch.bfloat16, device=device).normal_(0, 0.02,
                                                                              generator=gen)
    params, offset = [], 0
    for shape in shapes:
        n = math.prod(shape)
        params.append(torch.nn.Parameter(flat_p[offset:offset + n].view(shape)))
        offset += n
    fmt = {"exp_avg": StateFormat(torch.float8_e4m3fn, "stochastic"),
           "exp_avg_sq": StateFormat(torch.bfloat16, "stochastic")}
    # Flat gradient buffers (every p.grad a view into them): the layout the
    # host-streamed step of the e2e measurement loads into.
    opt = ZeroAdamW(params, lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.1,
                    state_format=fmt, seed=7, gather=gather, chunks=chunks,
                    grads="reduce_scatter")
    flat_g = opt.flat_grads(torch.bfloat16)
    flat_g.normal_(0, 1e-4, generator=gen)
    return opt, params, flat_p, flat_g, total


def time_steps(opt, steps, world, stream):
    """K steps bracketed by barrier + synchronize; CUDA events on the launch stream."""
    import torch

    barrier(world)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    torch.cuda.nvtx.range_push("timed")  # profilers can select the timed steps
    start.record(stream)
    for i in range(steps):
        opt.step()
        marks[i].record(stream)
    end.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier(world)
    total_ms = start.elapsed_time(end)
    per_step = [start.elapsed_time(marks[0])] + [
        marks[i - 1].elapsed_time(marks[i]) for i in range(1, steps)]
    return total_ms, per_step


def cpu_baseline(seconds):
    """The CPU oracle (a C port of the reference algorithm) on this host's cores,
    timed on a bounded sample of the same step: BF16 p/g, E4M3 SR m, BF16 SR v."""
    import numpy as np

    import oracle

    threads = oracle.cpu_threads()
    n = 1 << 22
    rng = np.random.default_rng(7)
    p = (rng.standard_normal(n, dtype=np.float32) * 0.02).view(np.uint32) >> 16
    g = (rng.standard_normal(n, dtype=np.float32) * 1e-4).view(np.uint32) >> 16
    p, g = p.astype(np.uint16), g.astype(np.uint16)
    m = np.zeros(n, np.uint8)
    v = np.zeros(n, np.uint16)

    def one_pass(step):
        oracle.adamw_(p, g, m, v, m_fmt=oracle.E4M3, m_rule=oracle.STOCHASTIC,
                      v_fmt=oracle.BF16, v_rule=oracle.STOCHASTIC, lr=3e-4, beta1=0.9,
                      beta2=0.999, eps=1e-8, weight_decay=0.1, step=step,
                      update_key=oracle.update_key(7, step, 0), threads=threads)

    one_pass(1)  # warm-up (page faults)
    passes, start = 0, time.perf_counter()
    while True:
        one_pass(passes + 2)
        passes += 1
        elapsed = time.perf_counter() - start
        if elapsed * threads >= seconds or elapsed >= seconds:
            break
    rate = passes * n / elapsed
    return {"value": rate, "unit": "params/s", "cores": threads, "kind": "port",
            "sample": f"{passes} passes over {n} elements (BF16 p/g, E4M3 SR m, BF16 SR v), "
                      f"{elapsed:.2f} s wall on {threads} threads"}


def e2e_run(opt, flat_p, flat_g, steps, world, total):
    """The step through the public API with host buffers (``ZeroAdamW.step_host``):
    per step each rank's BF16 gradient shard comes from pinned host memory and
    its updated BF16 parameter shard goes back to it, both streamed in tile
    chunks alongside the update (the optimizer states stay on the device)."""
    import torch

    n = opt.flat_numel(torch.bfloat16)
    host_g = torch.empty(n, dtype=torch.bfloat16, pin_memory=True)
    host_p = torch.empty(n, dtype=torch.bfloat16, pin_memory=True)
    host_g.copy_(flat_g[:n])
    shard = opt.local_numel()  # this rank's elements: what each copy moves
    opt.step_host(host_g, host_p)  # warm-up: streams and the chunk plan
    stream = torch.cuda.current_stream()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        opt.step_host(host_g, host_p)
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world) / steps
    return {"value": total / (ms / 1e3), "unit": "params/s", "ms_per_step": ms,
            "h2d_bytes_per_step": shard * 2, "d2h_bytes_per_step": shard * 2,
            "api": "ZeroAdamW.step_host (pinned host gradients in, parameters out)"}


def run_b200(args):
    import torch

    world, rank = init_distributed(args.gpus)
    peak, peak_source = measured_hbm_peak()
    opt, params, flat_p, flat_g, total = build_workload(world, rank, args.layers,
                                                        not args.no_embeddings, args.gather,
                                                        args.chunks)
    local = opt.local_numel()
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        opt.step()
    torch.cuda.synchronize()
    opt.timings.clear()
    with ClockSampler(torch.cuda.current_device()) as clocks:
        total_ms, per_step = time_steps(opt, args.steps, world, stream)
    total_ms = max_over_ranks(total_ms, world)
    ms = total_ms / args.steps
    kernel_ms = max_over_ranks(statistics.mean(t["update_ms"] for t in opt.timings), world)
    gather_ms = max_over_ranks(statistics.mean(t.get("gather_ms", 0.0) for t in opt.timings),
                               world)
    achieved = BYTES_PER_PARAM * local / (kernel_ms / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": total / (ms / 1e3), "unit": "params/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "llama3-8b AdamW-SR optimizer step (BASELINE config 4)"
                   + ("" if (args.layers, args.no_embeddings) == (32, False)
                      else f" reduced to {args.layers} layers, embeddings={not args.no_embeddings}"),
                   "params": total, "tensors": len(params), "param_dtype": "bf16",
                   "grad_dtype": "bf16", "exp_avg": "float8_e4m3fn stochastic",
                   "exp_avg_sq": "bfloat16 stochastic", "parallelism": f"zero1-dp{world}",
                   "gather": {"fused": "updated parameters stored into every peer replica by "
                                       "the step kernel (NVLink peer stores)",
                              "copy": "copy engines send each chunk of updated parameters to "
                                      "the peers while the next chunk is updated",
                              "nccl": "NCCL all-gather after the step",
                              "none": "one rank"}[opt.gather_mode],
                   "global_batch": None, "seq_len": None,
                   "l2": f"{BYTES_PER_PARAM * local / 1e9:.0f} GB moved per step and GPU, "
                         "larger than the 126 MB L2; no flush"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak,
                     "traffic": MEASURED_TRAFFIC_PER_PARAM * local,
                     "traffic_source": "ncu dram bytes per parameter of the 2-layer case, "
                                       "scaled to this launch",
                     "peak_source": peak_source,
                     "kernel": "srs::adamw_kernel<E4M3,BF16>", "kernel_ms": kernel_ms,
                     "bytes_per_param": BYTES_PER_PARAM, "params_per_launch": local},
        "gather_ms": gather_ms if world > 1 else 0.0,
        "step_ms_min": min(per_step), "gpu_launches": opt.launches_per_step() * args.steps,
        "clocks": clocks.report(),
    }
    if not args.no_e2e:
        line["e2e"] = e2e_run(opt, flat_p, flat_g, args.e2e_steps, world, total)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    if rank == 0:
        print(json.dumps(line), flush=True)
    opt.close()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def run_sgdm_gpt2(args):
    """Momentum SGD at the GPT-2-small shape on one GPU."""
    import torch

    from sr_states import StateFormat
    from sr_states.distributed import ZeroSGDM
    from sr_states.shapes import gpt2_small

    peak, peak_source = measured_hbm_peak()
    shapes = [s for _, s in gpt2_small()]
    total = sum(math.prod(s) for s in shapes)
    device = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=device).manual_seed(11)
    flat_p = torch.empty(total, dtype=torch.float32, device=device).normal_(0, 0.02,
                                                                             generator=gen)
    flat_g = torch.empty(total, dtype=torch.float32, device=device).normal_(0, 1e-3,
                                                                             generator=gen)
    params, offset = [], 0
    for shape in shapes:
        n = math.prod(shape)
        p = torch.nn.Parameter(flat_p[offset:offset + n].view(shape))
        p.grad = flat_g[offset:offset + n].view(shape)
        params.append(p)
        offset += n
    opt = ZeroSGDM(params, lr=1e-2, momentum=0.9,
                   state_format={"momentum_buffer": StateFormat(torch.bfloat16, "stochastic")},
                   seed=11)
    for _ in range(args.warmup):
        opt.step()
    torch.cuda.synchronize()
    opt.timings.clear()
    stream = torch.cuda.current_stream()
    with ClockSampler(torch.cuda.current_device()) as clocks:
        total_ms, per_step = time_steps(opt, args.steps, 1, stream)
    ms = total_ms / args.steps
    kernel_ms = statistics.mean(t["update_ms"] for t in opt.timings)
    bytes_per_param = 16  # read p (4), g (4), u (2); write p (4), u (2)
    achieved = bytes_per_param * total / (kernel_ms / 1e3) / 1e9
    print(json.dumps({
        "metric": "SGDM-SR step params/sec & HBM GB/s at GPT-2-small shape", "value":
        total / (ms / 1e3), "unit": "params/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "gpt2-small momentum SGD step (BASELINE config 3)",
                   "params": total, "tensors": len(params), "param_dtype": "f32",
                   "grad_dtype": "f32", "momentum_buffer": "bfloat16 stochastic",
                   "l2": f"{bytes_per_param * total / 1e9:.1f} GB moved per step, larger than "
                         "L2; no flush"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": None, "peak_source": peak_source,
                     "kernel": "srs::sgdm_kernel<BF16>", "kernel_ms": kernel_ms,
                     "bytes_per_param": bytes_per_param},
        "step_ms_min": min(per_step), "gpu_launches": opt.launches_per_step() * args.steps,
        "clocks": clocks.report()}), flush=True)


def run_cast(args):
    """The standalone cast of FP32 data: magnitudes 2^U(-20, 18)
    with random signs; one line per target format and rule at --cast-elems."""
    import torch

    from sr_states.cuda.cast import cast

    peak, peak_source = measured_hbm_peak()
    n = args.cast_elems
    device = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=device).manual_seed(7)
    x = torch.empty(n, device=device).uniform_(-20, 18, generator=gen).exp2_()
    x *= torch.empty(n, device=device).bernoulli_(0.5, generator=gen).mul_(2).sub_(1)
    stream = torch.cuda.current_stream()
    for dtype, size in ((torch.bfloat16, 2), (torch.float16, 2), (torch.float8_e4m3fn, 1),
                        (torch.float8_e5m2, 1)):
        for rule in ("stochastic", "nearest"):
            offset = 0
            for _ in range(args.warmup):
                cast(x, dtype=dtype, rounding=rule, seed=7, offset=offset)
                offset += n
            torch.cuda.synchronize()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(
                enable_timing=True)
            with ClockSampler(torch.cuda.current_device()) as clocks:
                torch.cuda.nvtx.range_push("timed")
                start.record(stream)
                for _ in range(args.steps):
                    out = cast(x, dtype=dtype, rounding=rule, seed=7, offset=offset)
                    offset += n
                end.record(stream)
                torch.cuda.nvtx.range_pop()
                torch.cuda.synchronize()
            ms = start.elapsed_time(end) / args.steps
            achieved = (4 + size) * n / (ms / 1e3) / 1e9
            print(json.dumps({
                "metric": "cast elements/sec & HBM GB/s", "value": n / (ms / 1e3),
                "unit": "elements/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": f"cast FP32 -> {str(dtype).split('.')[-1]} {rule} "
                                       "(BASELINE config 2)", "elements": n},
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak,
                             "unit": "GB/s", "frac": achieved / peak, "traffic": None,
                             "peak_source": peak_source, "kernel": "srs::cast_kernel",
                             "bytes_per_elem": 4 + size},
                "gpu_launches": args.steps, "clocks": clocks.report()}), flush=True)
            del out


def run_adamw_70b(args):
    """AdamW at the Llama-3-70B shape: 723 tensors,
    70,553,706,496 BF16 parameters in two groups (vectors: weight decay 0,
    AdamW step 5; matrices: weight decay 0.1, AdamW step 6), BF16 gradients,
    FP16 stochastic moments, seed 3.

    A replicated BF16 copy of the parameters (141 GB) plus full gradients do not
    fit in one B200, so every rank holds only its shard of the flat parameter
    buffer (in parameter-group order), of the gradients (as after a
    reduce-scatter) and of the states.  The step is the fused kernel over the
    rank's rows (one launch per group) followed by the all-gather of the
    updated parameters, in chunks through one reused 16 GB staging buffer (the
    way a sharded model streams its parameters); both are timed."""
    import torch
    import torch.distributed as dist

    from sr_states.cuda import _native
    from sr_states.cuda._fused import adamw_hparams, rng_words
    from sr_states.cuda._tables import DeviceTable, Update, build_table, upload
    from sr_states.shapes import llama3_70b

    world, rank = init_distributed(args.gpus)
    if world < 4:
        raise SystemExit("the 70B workload needs at least 4 GPUs (memory)")
    peak, peak_source = measured_hbm_peak()
    shapes = [s for _, s in llama3_70b()]
    ordered = [s for s in shapes if len(s) == 1] + [s for s in shapes if len(s) > 1]
    numels = [math.prod(s) for s in ordered]
    n_vectors = sum(1 for s in ordered if len(s) == 1)
    total = sum(numels)
    unit = world * 64
    shard = -(-total // unit) * unit // world
    lo, hi = rank * shard, (rank + 1) * shard
    device = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=device).manual_seed(3 + rank)
    p = torch.empty(shard, dtype=torch.bfloat16, device=device).normal_(0, 0.02, generator=gen)
    g = torch.empty(shard, dtype=torch.bfloat16, device=device).normal_(0, 1e-4, generator=gen)
    m = torch.zeros(shard, dtype=torch.float16, device=device)
    v = torch.zeros(shard, dtype=torch.float16, device=device)
    groups = ([], [])  # (vectors, matrices): updates of this rank's pieces
    offset = 0
    for index, n in enumerate(numels):
        a, b = max(lo, offset), min(hi, offset + n)
        if a < b:
            s, e = a - lo, b - lo
            groups[0 if index < n_vectors else 1].append(
                Update((p[s:e], g[s:e], m[s:e], v[s:e]), index, e - s, a - offset, None))
        offset += n
    tables = []
    for updates in groups:
        if updates:
            host = build_table(updates, [0] * len(updates), 2048)
            n_tiles = int(host["tile_begin"][-1] + -(-host["numel"][-1] // 2048))
            tables.append(DeviceTable(host, upload(host, device), len(host), n_tiles))
        else:
            tables.append(None)
    launcher = _native.launcher()
    launcher.check_device(device)
    chunk = min(shard, (16 * 10**9 // 2) // world)  # elements per rank and chunk
    staging = torch.empty(world * chunk, dtype=torch.bfloat16, device=device)
    stream = torch.cuda.current_stream()
    settings = ((0.0, 5), (0.1, 6))  # (weight decay, AdamW step at the first timed step)

    def one_step(i):
        rng = rng_words(3, 7 + i)
        for table, (wd, step) in zip(tables, settings):
            if table is not None:
                hp = adamw_hparams(3e-4, (0.9, 0.999), 1e-8, wd, (step + i,))
                launcher.adamw_multi(table, table.n_rows, table.n_tiles, 2, 1, 2, 1, hp, rng,
                                     stream.cuda_stream)
        marks[i][1].record(stream)
        for k in range(0, shard, chunk):
            c = min(chunk, shard - k)
            dist.all_gather_into_tensor(staging[:world * c], p[k:k + c])

    marks = [[torch.cuda.Event(enable_timing=True) for _ in range(3)]
             for _ in range(args.warmup + args.steps)]
    for i in range(args.warmup):
        marks[i][0].record(stream)
        one_step(i)
    torch.cuda.synchronize()
    with ClockSampler(torch.cuda.current_device()) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed")
        start.record(stream)
        for i in range(args.warmup, args.warmup + args.steps):
            marks[i][0].record(stream)
            one_step(i)
            marks[i][2].record(stream)
        end.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world) / args.steps
    timed = marks[args.warmup:]
    update_ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b, _ in timed), world)
    gather_ms = max_over_ranks(statistics.mean(b.elapsed_time(c) for _, b, c in timed), world)
    bytes_per_param = 14  # read p 2, g 2, m 2, v 2; write p 2, m 2, v 2
    achieved = bytes_per_param * shard / (update_ms / 1e3) / 1e9
    line = {
        "metric": "AdamW-SR step params/sec & HBM GB/s at 70B shape", "value": total / (ms / 1e3),
        "unit": "params/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": "llama3-70b AdamW-SR optimizer step (BASELINE config 5)",
                   "params": total, "tensors": len(ordered), "param_dtype": "bf16",
                   "grad_dtype": "bf16", "exp_avg": "float16 stochastic",
                   "exp_avg_sq": "float16 stochastic",
                   "groups": "vectors wd 0 (AdamW step 5), matrices wd 0.1 (AdamW step 6)",
                   "parallelism": f"sharded parameters, gradients and states over {world} GPUs; "
                                  "NCCL all-gather of the parameters in chunks through a "
                                  f"{staging.numel() * 2 / 1e9:.0f} GB staging buffer",
                   "l2": f"{bytes_per_param * shard / 1e9:.0f} GB moved per step and GPU; no flush"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": None, "peak_source": peak_source,
                     "kernel": "srs::adamw_kernel<F16,F16>", "kernel_ms": update_ms,
                     "bytes_per_param": bytes_per_param, "params_per_launch": shard},
        "gather_ms": gather_ms, "gpu_launches": sum(t is not None for t in tables) * args.steps,
        "clocks": clocks.report()}
    if rank == 0:
        print(json.dumps(line), flush=True)
    dist.destroy_process_group()


def run_reference(args):
    """The reference arm: the CPU restatement of the reference algorithm (the reference
    itself is Python on PyTorch's CPU kernels and does not travel to this box) on all
    host cores; every step is a bounded sample of the same workload."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    samples = [cpu_baseline(args.cpu_seconds / max(args.steps, 1))
               for _ in range(args.warmup + args.steps)][args.warmup:]
    value = statistics.median(s["value"] for s in samples)
    base = dict(samples[-1], value=value)
    print(json.dumps({
        "metric": METRIC, "impl": "reference", "value": value, "unit": "params/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 8030261248 / value * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "llama3-8b AdamW-SR optimizer step (BASELINE config 4)",
                   "params": 8030261248, "tensors": 291, "param_dtype": "bf16",
                   "grad_dtype": "bf16", "exp_avg": "float8_e4m3fn stochastic",
                   "exp_avg_sq": "bfloat16 stochastic", "parallelism": "host cores",
                   "global_batch": None, "seq_len": None,
                   "timing": "each step a bounded sample of the workload, scaled to its "
                             "8,030,261,248 parameters (see cpu_baseline.sample)"},
        "cpu_baseline": base,
        "e2e": {"value": value, "unit": "params/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}), flush=True)


def main(argv=None):
    args = parse_args(argv)
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "sgdm-gpt2":
        run_sgdm_gpt2(args)
    elif args.workload == "cast":
        run_cast(args)
    elif args.workload == "adamw-70b":
        run_adamw_70b(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
