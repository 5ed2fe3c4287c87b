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
    --workload nvlink-exchange
                           the fused step's peer stores in isolation: one
                           process, GPU 0 updating and storing into a replica
                           on GPU 1 (for NVLink counters; needs two GPUs)
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
# (dram__bytes_read.sum + dram__bytes_write.sum = 5.188656 GB over the 436,228,096
# parameters of the 2-layer profiling case; profiles/adamw_kernel_llama3-8b.md).
# Traffic grows in proportion to the parameters, so a full launch moves this
# many bytes per parameter.
MEASURED_TRAFFIC_PER_PARAM = 11.894
FALLBACK_HBM_GBS = 6650.0
# BASELINE config 4 hyperparameters.
LR, BETAS, EPS, WEIGHT_DECAY, SEED = 3e-4, (0.9, 0.999), 1e-8, 0.1, 7
# Measured peer copy bandwidth per direction and GPU over NVLink 5 on this pool
# (copy engines); nominal 900 GB/s.
NVLINK_PEER_GBS = 770.0


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
    parser.add_argument("--layers-70b", type=int, default=80,
                        help="decoder layers of the Llama-3-70B shape (config 5; fewer only to "
                             "check the workload on fewer GPUs)")
    parser.add_argument("--no-embeddings", action="store_true",
                        help="drop the two 128256x4096 matrices (profiling case)")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-secondary", action="store_true",
                        help="skip the config-3 SGDM and config-2 cast lines of the default run")
    parser.add_argument("--workload", choices=("adamw-8b", "sgdm-gpt2", "cast", "adamw-70b",
                                               "nvlink-exchange"),
                        default="adamw-8b")
    parser.add_argument("--exchange-elems", type=int, default=1 << 26,
                        help="parameters of the nvlink-exchange workload")
    parser.add_argument("--gather", choices=("auto", "fused", "copy", "nccl", "multicast",
                                             "hybrid"),
                        default="auto",
                        help="how the sharded step reassembles the parameters at N>1")
    parser.add_argument("--chunks", type=int, default=32,
                        help="tile chunks of the pipelined exchange (--gather copy, hybrid)")
    parser.add_argument("--copy-peers", type=int, default=1,
                        help="peers served by the copy engines (--gather hybrid)")
    parser.add_argument("--copy-streams", type=int, default=None,
                        help="copy streams of the copy-engine exchange (default: one per peer)")
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


def box_copy_gbs(world):
    """This GPU's own device-copy rate (slowest rank): one 4 GiB FP32 buffer
    copied into another (32x the L2), best of 5, CUDA events; bytes read plus
    written per second.  Context for box-to-box differences of the kernel's
    rate; the roofline's peak stays the pool's measured copy bandwidth."""
    import torch

    n = 1 << 30
    src = torch.ones(n, dtype=torch.float32, device="cuda")
    dst = torch.empty_like(src)
    stream = torch.cuda.current_stream()
    for _ in range(2):
        dst.copy_(src)
    best = float("inf")
    for _ in range(5):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        dst.copy_(src)
        end.record(stream)
        end.synchronize()
        best = min(best, start.elapsed_time(end))
    del src, dst
    torch.cuda.empty_cache()
    return -max_over_ranks(-(2 * 4 * n / (best / 1e3) / 1e9), world)


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

def build_workload(world, rank, layers=32, embeddings=True, gather="auto", chunks=32,
                   copy_peers=1, copy_streams=None):
    """Flat BF16 parameter and gradient buffers holding the 291 tensors; the
    optimizer (ZeRO-1 when world > 1) over views of them."""
    import torch

    from sr_states import StateFormat
    from sr_states.distributed import ZeroAdamW
    from sr_states.shapes import llama3_8b

    named = [(name, s) for name, s in llama3_8b()
             if (embeddings or name not in ("embed_tokens", "lm_head"))
             and not (name.startswith("layers.") and int(name.split(".")[1]) >= layers)]
    names, shapes = [n for n, _ in named], [s for _, s in named]
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
    opt = ZeroAdamW(params, lr=LR, betas=BETAS, eps=EPS, weight_decay=WEIGHT_DECAY,
                    state_format=fmt, seed=SEED, gather=gather, chunks=chunks,
                    grads="reduce_scatter", record_timings=True, copy_peers=copy_peers,
                    copy_streams=copy_streams)
    flat_g = opt.flat_grads(torch.bfloat16)
    flat_g.normal_(0, 1e-4, generator=gen)
    return opt, names, params, flat_p, flat_g, total


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
    n = 1 << 24
    rng = np.random.default_rng(7)
    p = (rng.standard_normal(n, dtype=np.float32) * 0.02).view(np.uint32) >> 16
    g = (rng.standard_normal(n, dtype=np.float32) * 1e-4).view(np.uint32) >> 16
    p, g = p.astype(np.uint16), g.astype(np.uint16)
    m = np.zeros(n, np.uint8)
    v = np.zeros(n, np.uint16)

    def one_pass(step):
        oracle.adamw_(p, g, m, v, m_fmt=oracle.E4M3, m_rule=oracle.STOCHASTIC,
                      v_fmt=oracle.BF16, v_rule=oracle.STOCHASTIC, lr=LR, beta1=BETAS[0],
                      beta2=BETAS[1], eps=EPS, weight_decay=WEIGHT_DECAY, step=step,
                      update_key=oracle.update_key(SEED, step, 0), threads=threads)

    one_pass(1)  # warm-up (page faults)
    rates = []
    start = time.perf_counter()
    while True:
        t = time.perf_counter()
        one_pass(len(rates) + 2)
        rates.append(n / (time.perf_counter() - t))
        elapsed = time.perf_counter() - start
        if elapsed >= seconds:
            break
    return {"value": statistics.median(rates), "unit": "params/s", "cores": threads,
            "kind": "port",
            "sample": f"median of {len(rates)} passes over {n} elements (BF16 p/g, E4M3 SR m, "
                      f"BF16 SR v) of the C restatement, {elapsed:.2f} s wall on {threads} "
                      "threads"}


REFERENCE_DIR = ROOT / "baseline" / "_ref"
REFERENCE_SAMPLE = 1 << 24  # elements of the reference arm's sample tensor


def reference_cpu_steps(steps, warmup):
    """The reference's own CPU path: ``AdamWReferenceSR.step`` of the unmodified
    reference package (installed in baseline/_ref) on one 2^24-element tensor
    with the config's formats (BF16 parameter and gradient, E4M3 stochastic
    exp_avg, BF16 stochastic exp_avg_sq) and hyperparameters, all host threads.
    Returns the per-step rates (params/s) and the thread count, or None when the
    reference is not installed.  Must run before anything imports this
    repository's own ``sr_states`` (the packages share the name)."""
    if not (REFERENCE_DIR / "sr_states").is_dir():
        return None
    ours = str((ROOT / "stochastic-rounding-pytorch_b200").resolve())
    sys.path[:] = [x for x in sys.path if str(Path(x or ".").resolve()) != ours]
    sys.path.insert(0, str(REFERENCE_DIR))
    import torch

    import sr_states

    if Path(sr_states.__file__).resolve().parents[1] != REFERENCE_DIR.resolve():
        raise RuntimeError(f"expected the reference's sr_states, imported {sr_states.__file__}")
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(SEED)
    p = torch.nn.Parameter((torch.randn(REFERENCE_SAMPLE, generator=gen) * 0.02)
                           .to(torch.bfloat16))
    p.grad = (torch.randn(REFERENCE_SAMPLE, generator=gen) * 1e-4).to(torch.bfloat16)
    fmt = {"exp_avg": sr_states.StateFormat(torch.float8_e4m3fn, "stochastic"),
           "exp_avg_sq": sr_states.StateFormat(torch.bfloat16, "stochastic")}
    opt = sr_states.AdamWReferenceSR([p], lr=LR, betas=BETAS, eps=EPS,
                                     weight_decay=WEIGHT_DECAY, state_format=fmt, seed=SEED)
    rates = []
    for i in range(warmup + steps):
        t = time.perf_counter()
        opt.step()
        dt = time.perf_counter() - t
        if i >= warmup:
            rates.append(REFERENCE_SAMPLE / dt)
    return rates, torch.get_num_threads()


def reference_baseline_entry(rates, threads):
    return {"value": statistics.median(rates), "unit": "params/s", "cores": threads,
            "kind": "reference",
            "sample": f"median of {len(rates)} steps of the reference's AdamWReferenceSR.step "
                      f"(unmodified package, baseline/_ref) on one {REFERENCE_SAMPLE}-element "
                      "BF16 parameter with E4M3/BF16 stochastic states, "
                      f"{sum(REFERENCE_SAMPLE / r for r in rates):.1f} s on {threads} threads; "
                      "scaled to the config's parameters",
            "spread": [min(rates), max(rates)]}


def cpu_reference_subprocess(args):
    """The reference CPU baseline measured in a fresh interpreter (this process
    already imported this repository's ``sr_states``): the reference arm itself,
    a few steps."""
    import subprocess

    if not (REFERENCE_DIR / "sr_states").is_dir():
        return None
    env = {k: v for k, v in os.environ.items()
           if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT")}
    out = subprocess.run([sys.executable, str(Path(__file__).resolve()), "--impl", "reference",
                          "--steps", "5", "--warmup", "1"], env=env, capture_output=True,
                         text=True, timeout=900)
    if out.returncode != 0:
        return None
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    if not lines:
        return None
    entry = json.loads(lines[-1]).get("cpu_baseline")
    if entry is not None:
        entry.pop("port", None)
    return entry


# ----------------------------------------------------------- verification --

VERIFY_WINDOW = 2048  # elements per sampled window


def sample_windows(names, shapes, world, shard):
    """Flat element windows [a, b) of the BF16 buffer whose update is checked:
    both sides of every shard boundary, the head and tail of embed_tokens and
    lm_head, the first layer's and the final RMSNorm vectors, and the middle of
    a large matrix.  Merged where they overlap."""
    offsets, at = {}, 0
    for name, shape in zip(names, shapes):
        offsets[name] = (at, math.prod(shape))
        at += math.prod(shape)
    total, half = at, VERIFY_WINDOW // 2
    wanted = [(k * shard - half, k * shard + half) for k in range(1, world)]
    for name in ("embed_tokens", "lm_head"):
        if name in offsets:
            start, n = offsets[name]
            wanted += [(start, start + VERIFY_WINDOW), (start + n - VERIFY_WINDOW, start + n)]
    for name in ("layers.0.input_layernorm", "norm"):
        if name in offsets:
            start, n = offsets[name]
            wanted.append((start, start + n))
    if "layers.0.gate_proj" in offsets:
        start, n = offsets["layers.0.gate_proj"]
        wanted.append((start + n // 2 - half, start + n // 2 + half))
    merged = []
    for a, b in sorted((max(0, a), min(total, b)) for a, b in wanted):
        if a >= b:
            continue
        if merged and a <= merged[-1][1]:
            merged[-1] = (merged[-1][0], max(b, merged[-1][1]))
        else:
            merged.append((a, b))
    return merged, offsets


def buffer_digest(buffer, n):
    """Position-weighted checksum of the first n elements of a 16-bit buffer:
    (sum of words, sum of (i+1) * word) mod 2^64, on the device in chunks."""
    import torch

    words = buffer.view(torch.int16)
    chunk = 1 << 26
    index = torch.arange(1, chunk + 1, dtype=torch.int64, device=buffer.device)
    s1 = torch.zeros((), dtype=torch.int64, device=buffer.device)
    s2 = torch.zeros((), dtype=torch.int64, device=buffer.device)
    for a in range(0, n, chunk):
        x = words[a:min(n, a + chunk)].to(torch.int64)
        s1 += x.sum()
        s2 += (x * (index[:x.numel()] + a)).sum()
    return int(s1.item()), int(s2.item())


def verify_step(opt, names, params, world, rank):
    """One more optimizer step (untimed), checked two ways:

    * every rank's replica of the flat BF16 parameters has the same digest
      (the exchange delivered every shard everywhere);
    * rank 0 recomputes sampled windows with the CPU oracle (the checker of the
      tests) from the inputs of that step, gathered from the ranks that own
      their optimizer states, and compares the parameter bytes of its own
      replica and the states' bytes of their owners.
    """
    import numpy as np
    import torch
    import torch.distributed as dist

    from sr_states.distributed import shard_sizes

    total = opt.flat_numel(torch.bfloat16)
    shard = shard_sizes(total, world)
    windows, offsets = sample_windows(names, [p.shape for p in params], world, shard)
    index_of = {name: i for i, name in enumerate(names)}
    segments = []  # (param index, lo, hi) within the parameter
    for a, b in windows:
        for name, (start, n) in offsets.items():
            lo, hi = max(a, start) - start, min(b, start + n) - start
            if lo < hi:
                segments.append((index_of[name], lo, hi))

    def bits(t, width):  # a copy, never a view of live memory
        return t.detach().contiguous().view(width).cpu().numpy().copy()

    def capture(with_params):
        out = {}
        for k, (i, lo, hi) in enumerate(segments):
            p = params[i]
            entry = {}
            if with_params:
                entry["p"] = bits(p.detach().reshape(-1)[lo:hi], torch.int16).view(np.uint16)
                entry["g"] = bits(p.grad.reshape(-1)[lo:hi], torch.int16).view(np.uint16)
            run = opt.local_run(p)
            if run is not None and max(lo, run[0]) < min(hi, run[1]):
                a, b = max(lo, run[0]), min(hi, run[1])
                st = opt.state[p]
                entry["run"] = (a, b)
                entry["m"] = bits(st["exp_avg"][a - run[0]:b - run[0]], torch.uint8)
                entry["v"] = bits(st["exp_avg_sq"][a - run[0]:b - run[0]],
                                  torch.int16).view(np.uint16)
                entry["step"] = int(st.get("step", 0))
            out[k] = entry
        return out

    sync = torch.cuda.synchronize if torch.cuda.is_available() else (lambda: None)
    sync()
    before = capture(rank == 0)
    opt.step()
    sync()
    after = capture(rank == 0)
    digest = buffer_digest(opt.flat_params(torch.bfloat16), total)
    rng_step = int(opt.param_groups[0]["sr_step"])
    gathered = [None] * world
    if world > 1:
        dist.all_gather_object(gathered, (digest, before, after))
    else:
        gathered = [(digest, before, after)]
    if rank != 0:
        return None

    import oracle

    replicas_equal = all(d == gathered[0][0] for d, _, _ in gathered)
    mismatched, checked = 0, 0
    for k, (i, lo, hi) in enumerate(segments):
        p = before[k]["p"].copy()
        g = before[k]["g"]
        m = np.zeros(hi - lo, np.uint8)
        v = np.zeros(hi - lo, np.uint16)
        m_after = np.zeros(hi - lo, np.uint8)
        v_after = np.zeros(hi - lo, np.uint16)
        owned = np.zeros(hi - lo, bool)
        steps = set()
        for _, b_r, a_r in gathered:
            if "run" in b_r[k]:
                a, b = b_r[k]["run"]
                m[a - lo:b - lo], v[a - lo:b - lo] = b_r[k]["m"], b_r[k]["v"]
                m_after[a - lo:b - lo], v_after[a - lo:b - lo] = a_r[k]["m"], a_r[k]["v"]
                owned[a - lo:b - lo] = True
                steps.add(a_r[k]["step"])
        if not owned.all() or len(steps) != 1:
            mismatched += 1 << 30  # a window nobody (or two steps) covered: fail loudly
            continue
        oracle.adamw_(p, g.copy(), m, v, m_fmt=oracle.E4M3, m_rule=oracle.STOCHASTIC,
                      v_fmt=oracle.BF16, v_rule=oracle.STOCHASTIC, lr=LR, beta1=BETAS[0],
                      beta2=BETAS[1], eps=EPS, weight_decay=WEIGHT_DECAY, step=steps.pop(),
                      update_key=oracle.update_key(SEED, rng_step, i), offset=lo)
        mismatched += int(np.count_nonzero(p.view(np.uint8) != after[k]["p"].view(np.uint8)))
        mismatched += int(np.count_nonzero(m != m_after))
        mismatched += int(np.count_nonzero(v.view(np.uint8) != v_after.view(np.uint8)))
        checked += hi - lo
    return {"replicas_equal": replicas_equal, "digest": list(gathered[0][0]),
            "windows": len(windows), "rows": len(segments), "elements": checked,
            "mismatched_bytes": mismatched, "rng_step": rng_step,
            "checker": "CPU oracle (tests' checker) on sampled windows: both sides of every "
                       "shard boundary, head and tail of embed_tokens and lm_head, two RMSNorm "
                       "vectors, the middle of a matrix; p from rank 0's replica, m and v "
                       "from their owners"}


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
    link = pcie_rates(host_g, host_p, flat_g, world)
    moved = shard * 2 / (ms / 1e3) / 1e9  # each direction
    return {"value": total / (ms / 1e3), "unit": "params/s", "ms_per_step": ms,
            "h2d_bytes_per_step": shard * 2, "d2h_bytes_per_step": shard * 2,
            "pcie": {"achieved_gbs_per_direction": moved, **link,
                     "frac": moved / min(link["h2d_gbs"], link["d2h_gbs"]),
                     "how": "peak: 2 GiB pinned copies in both directions at once on two "
                            "streams, CUDA events, best of 3, all ranks copying together"},
            "api": "ZeroAdamW.step_host (pinned host gradients in, parameters out)" + (
                f"; each of the {world} ranks loads its own gradient shard and sends back its "
                "own updated parameter shard (bytes above are per rank)" if world > 1 else "")}


def pcie_rates(host_g, host_p, device_buffer, world):
    """Host<->device copy bandwidth in each direction with both running at once
    (as in the host-streamed step), from this rank's pinned buffers."""
    import torch

    n = min(host_g.numel(), host_p.numel(), device_buffer.numel(), 1 << 30)  # 2 GiB of BF16
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    scratch = torch.empty(n, dtype=torch.bfloat16, device=device_buffer.device)
    best = (0.0, 0.0)
    for _ in range(3):
        barrier(world)
        torch.cuda.synchronize()
        marks = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        marks[0].record(up)
        marks[2].record(down)
        with torch.cuda.stream(up):
            scratch.copy_(host_g[:n], non_blocking=True)
        with torch.cuda.stream(down):
            host_p[:n].copy_(device_buffer[:n], non_blocking=True)
        marks[1].record(up)
        marks[3].record(down)
        torch.cuda.synchronize()
        rates = (2 * n / (marks[0].elapsed_time(marks[1]) / 1e3) / 1e9,
                 2 * n / (marks[2].elapsed_time(marks[3]) / 1e3) / 1e9)
        best = max(best, rates, key=lambda r: min(r))
    del scratch
    return {"h2d_gbs": best[0], "d2h_gbs": best[1]}


def split_phase(opt, steps, world, stream):
    """At N > 1: the same steps with the update and the exchange as separate
    launches (the NCCL all-gather after the update), so the update alone and the
    exchange alone are timed.  Nothing is skipped: the parameters that leave
    these steps are the same as the fused exchange's."""
    import torch

    connected = opt.gather_mode
    opt.set_gather_mode("nccl")
    try:
        opt.step()  # warm-up of the NCCL path
        torch.cuda.synchronize()
        opt.timings.clear()
        time_steps(opt, steps, world, stream)
        timings = list(opt.timings)
        opt.timings.clear()
    finally:
        opt.set_gather_mode(connected)
    return (max_over_ranks(statistics.mean(t["update_ms"] for t in timings), world),
            max_over_ranks(statistics.mean(t["gather_ms"] for t in timings), world))


def secondary_workloads(args):
    """BASELINE configs 3 and 2 measured in the same run as the headline (one
    GPU, after it): the GPT-2-small SGDM step and the 2^30-element casts, each
    with its roofline and clocks, so their numbers come from the same timed
    command as the headline."""
    sub = argparse.Namespace(**{**vars(args), "steps": max(args.steps, 10),
                                "warmup": max(args.warmup, 3)})
    keep = ("value", "unit", "ms_per_step", "step_ms_min", "roofline", "clocks", "gpu_launches")
    sgdm = measure_sgdm_gpt2(sub)
    casts = measure_casts(sub)
    return {
        "sgdm_gpt2": {"workload": sgdm["config"]["workload"], **{k: sgdm[k] for k in keep
                                                                  if k in sgdm}},
        "casts": [{"workload": c["config"]["workload"], "elements": c["config"]["elements"],
                   **{k: c[k] for k in keep if k in c}} for c in casts]}


def run_b200(args):
    import torch

    world, rank = init_distributed(args.gpus)
    peak, peak_source = measured_hbm_peak()
    opt, names, params, flat_p, flat_g, total = build_workload(
        world, rank, args.layers, not args.no_embeddings, args.gather, args.chunks,
        args.copy_peers, args.copy_streams)
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
    step_kernel_ms = max_over_ranks(statistics.mean(t["update_ms"] for t in opt.timings), world)
    barrier_ms = max_over_ranks(statistics.mean(t.get("gather_ms", 0.0) for t in opt.timings),
                                world)
    opt.timings.clear()
    if world > 1:
        update_ms, nccl_ms = split_phase(opt, args.steps, world, stream)
    else:
        update_ms, nccl_ms = step_kernel_ms, None
    box_copy = box_copy_gbs(world)
    achieved = BYTES_PER_PARAM * local / (update_ms / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": total / (ms / 1e3), "unit": "params/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "dtype_meaning": "arithmetic of the update (FP32 math); storage: BF16 parameters and "
                         "gradients, FP8 E4M3 exp_avg, BF16 exp_avg_sq",
        "data": "synthetic",
        "config": {"workload": "llama3-8b AdamW-SR optimizer step (BASELINE config 4)"
                   + ("" if (args.layers, args.no_embeddings) == (32, False)
                      else f" reduced to {args.layers} layers, embeddings={not args.no_embeddings}"),
                   "params": total, "tensors": len(params), "param_dtype": "bf16",
                   "grad_dtype": "bf16", "exp_avg": "float8_e4m3fn stochastic",
                   "exp_avg_sq": "bfloat16 stochastic", "parallelism": f"zero1-dp{world}",
                   "gather": {"fused": "updated parameters stored into every peer replica by "
                                       "the step kernel (NVLink peer stores)",
                              "hybrid": "the step's tile ranges store the updated parameters "
                                        "into all peer replicas but one; the copy engines send "
                                        "each finished range to that one",
                              "multicast": "each updated vector stored once by the step kernel "
                                           "to an NVLink multicast address (multimem.st); "
                                           "NVSwitch delivers it to every replica",
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
                     "kernel": "srs::adamw_kernel<E4M3,BF16>", "kernel_ms": update_ms,
                     "timed": "the update launch alone" + (
                         " (from the steps whose exchange is a separate NCCL all-gather)"
                         if world > 1 else ""),
                     "bytes_per_param": BYTES_PER_PARAM, "params_per_launch": local,
                     "box_copy_gbs": box_copy,
                     "frac_of_box_copy": achieved / box_copy,
                     "box_copy_how": "torch device copy of a 4 GiB FP32 buffer on this GPU "
                                     "after the timed steps, best of 5, CUDA events (slowest "
                                     "rank); context, not the peak"},
        "step_ms_min": min(per_step), "gpu_launches": opt.launches_per_step() * args.steps,
        "clocks": clocks.report(),
    }
    if world > 1:
        received = (world - 1) * local * 2  # BF16 bytes every GPU receives per step
        line["exchange"] = {
            "mechanism": opt.gather_mode, "bytes_received_per_gpu": received,
            "step_kernel_ms": step_kernel_ms, "barriers_ms": barrier_ms,
            "receive_gbs": received / (ms / 1e3) / 1e9,
            "bound_gbs": NVLINK_PEER_GBS,
            "frac": received / (ms / 1e3) / 1e9 / NVLINK_PEER_GBS,
            "bound_source": "measured peer copy per direction and GPU (copy engines); "
                            "nominal NVLink 5: 900 GB/s",
            "receive_bound_ms": received / (NVLINK_PEER_GBS * 1e9) * 1e3,
            "update_alone_ms": update_ms, "nccl_allgather_ms": nccl_ms,
            "nccl_allgather_gbs": received / (nccl_ms / 1e3) / 1e9}
    line["verify"] = verify_step(opt, names, params, world, rank)
    if rank != 0:
        line.pop("verify")
    if (world >= 4 or (world > 1 and args.layers_70b < 80)) and not args.no_secondary:
        # BASELINE config 5 (70B, everything sharded) where every rank has room
        # (a reduced layer count lets two GPUs check this path).
        if adamw_70b_fits(world, args.layers_70b):
            sub = argparse.Namespace(**{**vars(args), "steps": min(args.steps, 5),
                                        "warmup": min(args.warmup, 2)})
            big = measure_adamw_70b(sub, world, rank, args.layers_70b)
            line["secondary"] = {"adamw_70b": {
                "workload": big["config"]["workload"], "parallelism": big["config"]["parallelism"],
                **{k: big[k] for k in ("value", "unit", "ms_per_step", "roofline", "gather_ms",
                                       "clocks", "gpu_launches")}}}
        else:
            line["secondary"] = {"adamw_70b": "skipped: not enough free memory on every rank"}
    if not args.no_e2e:
        line["e2e"] = e2e_run(opt, flat_p, flat_g, args.e2e_steps, world, total)
    if world == 1 and not args.no_secondary:
        line["secondary"] = secondary_workloads(args)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_reference_subprocess(args) or cpu_baseline(args.cpu_seconds)
        line["cpu_baseline"]["port"] = cpu_baseline(min(args.cpu_seconds, 4.0))
    if rank == 0:
        print(json.dumps(line), flush=True)
    opt.close()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def run_sgdm_gpt2(args):
    print(json.dumps(measure_sgdm_gpt2(args)), flush=True)


def measure_sgdm_gpt2(args):
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
                   seed=11, record_timings=True)
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
    opt.close()
    return {
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
        "clocks": clocks.report()}


def run_cast(args):
    for line in measure_casts(args):
        print(json.dumps(line), flush=True)


def measure_casts(args):
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
    lines = []
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
            lines.append({
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
                "gpu_launches": args.steps, "clocks": clocks.report()})
            del out
    del x
    return lines


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
    import torch.distributed as dist

    world, rank = init_distributed(args.gpus)
    if not adamw_70b_fits(world, args.layers_70b):
        raise SystemExit("not enough device memory on every rank for this 70B shard "
                         "(the full model needs at least 4 GPUs)")
    line = measure_adamw_70b(args, world, rank, args.layers_70b)
    if rank == 0:
        print(json.dumps(line), flush=True)
    dist.destroy_process_group()


ADAMW_70B_BYTES_PER_PARAM = 8  # per rank: BF16 parameter and gradient, FP16 moments


def llama3_70b_shapes(layers=80):
    """The Llama-3-70B parameter shapes, optionally with fewer decoder layers."""
    from sr_states.shapes import _llama

    return [s for _, s in _llama(layers, 8192, 8 * 128, 28672)]


def adamw_70b_fits(world, layers=80):
    """Whether every rank has room for its 70B shard (parameters, gradients and
    FP16 states of the model's parameters / world, plus the 16 GB staging
    buffer and 8 GB of headroom); agreed over the ranks."""
    import torch
    import torch.distributed as dist

    total = sum(math.prod(s) for s in llama3_70b_shapes(layers))
    need = total // world * ADAMW_70B_BYTES_PER_PARAM + 24 * 10**9
    free = torch.tensor([torch.cuda.mem_get_info()[0]], dtype=torch.int64, device="cuda")
    dist.all_reduce(free, op=dist.ReduceOp.MIN)
    return int(free.item()) >= need


def measure_adamw_70b(args, world, rank, layers=80):
    import torch
    import torch.distributed as dist

    from sr_states.cuda import _native
    from sr_states.cuda._fused import adamw_hparams, rng_words
    from sr_states.cuda._tables import DeviceTable, Update, build_table, upload

    peak, peak_source = measured_hbm_peak()
    shapes = llama3_70b_shapes(layers)
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
        "config": {"workload": "llama3-70b AdamW-SR optimizer step (BASELINE config 5)"
                               + ("" if layers == 80 else f" reduced to {layers} layers"),
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
    del p, g, m, v, staging, tables
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return line


def run_nvlink_exchange(args):
    """The fused exchange of a sharded AdamW step in isolation, in ONE process
    driving two GPUs: GPU 0 updates --exchange-elems parameters (config-4
    formats) and stores every updated BF16 vector both locally and into a
    replica on GPU 1 over NVLink (peer stores from the step kernel, as ZeRO-1's
    fused gather does at N=2).  One process, so a profiler can capture the
    kernel's NVLink counters on GPU 0 alone.  Prints the kernel time, the
    NVLink bytes it must send and the rate, and checks the replica."""
    import torch
    from cuda.bindings import runtime as cudart

    from sr_states.cuda import _native
    from sr_states.cuda._fused import adamw_hparams, rng_words
    from sr_states.cuda._tables import DeviceTable, Update, build_table, upload

    if torch.cuda.device_count() < 2:
        raise SystemExit("--workload nvlink-exchange needs two GPUs in one process")
    src, dst = torch.device("cuda", 0), torch.device("cuda", 1)
    torch.cuda.set_device(src)
    err, = cudart.cudaSetDevice(0)[:1]
    err2, = cudart.cudaDeviceEnablePeerAccess(1, 0)[:1]
    if int(err) != 0 or int(err2) not in (0, int(cudart.cudaError_t.cudaErrorPeerAccessAlreadyEnabled)):
        raise SystemExit(f"peer access 0 -> 1 unavailable ({err}, {err2})")
    n = args.exchange_elems
    gen = torch.Generator(device=src).manual_seed(SEED)
    p = torch.empty(n, dtype=torch.bfloat16, device=src).normal_(0, 0.02, generator=gen)
    g = torch.empty(n, dtype=torch.bfloat16, device=src).normal_(0, 1e-4, generator=gen)
    m = torch.zeros(n, dtype=torch.float8_e4m3fn, device=src)
    v = torch.zeros(n, dtype=torch.bfloat16, device=src)
    replica = torch.zeros(n, dtype=torch.bfloat16, device=dst)
    host = build_table([Update((p, g, m, v), 0, n, 0, 1)], [0], 2048)
    n_tiles = int(-(-n // 2048))
    table = DeviceTable(host, upload(host, src), 1, n_tiles)
    peers = _native.SrsPeers()
    peers.n_peers = 1
    peers.delta_bf16[0] = replica.data_ptr() - p.data_ptr()
    launcher = _native.launcher()
    launcher.check_device(src)
    stream = torch.cuda.current_stream(src)

    def launch(i):
        hp = adamw_hparams(LR, BETAS, EPS, WEIGHT_DECAY, (i + 1,))
        launcher.adamw_multi(table, 1, n_tiles, 3, 1, 1, 1, hp, rng_words(SEED, i + 1),
                             stream.cuda_stream, peers=peers)

    for i in range(args.warmup):
        launch(i)
    torch.cuda.synchronize(src)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(args.warmup, args.warmup + args.steps):
        launch(i)
    end.record(stream)
    torch.cuda.synchronize(src)
    torch.cuda.synchronize(dst)
    ms = start.elapsed_time(end) / args.steps
    same = bool(torch.equal(replica.view(torch.int16).cpu(), p.view(torch.int16).cpu()))
    print(json.dumps({
        "metric": "fused AdamW step + peer stores, one GPU to one peer over NVLink",
        "value": 2 * n / (ms / 1e3) / 1e9, "unit": "GB/s NVLink (BF16 bytes stored to the peer)",
        "n_gpus": 2, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "data": "synthetic",
        "config": {"workload": "nvlink-exchange", "elements": n, "formats": "BF16 p/g, E4M3 SR "
                   "m, BF16 SR v", "hbm_bytes_per_launch": BYTES_PER_PARAM * n,
                   "nvlink_bytes_per_launch": 2 * n},
        "hbm_gbs": BYTES_PER_PARAM * n / (ms / 1e3) / 1e9, "replica_equal": same,
        "gpu_launches": args.steps}), flush=True)


def run_reference(args):
    """The reference arm: the reference's own CPU implementation of the step
    (``AdamWReferenceSR.step`` of the unmodified package in baseline/_ref) on
    all host cores; every step is a 2^24-element sample of the workload, the
    rate scaled to its 8,030,261,248 parameters.  Without the installed
    reference, the C restatement of the algorithm (the tests' oracle) stands in,
    labelled ``kind: port``.  Under torchrun only rank 0 runs."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    measured = reference_cpu_steps(args.steps, args.warmup)
    if measured is not None:
        base = reference_baseline_entry(*measured)
    else:
        samples = [cpu_baseline(max(1.0, args.cpu_seconds / max(args.steps, 1)))
                   for _ in range(args.steps)]
        base = dict(samples[-1], value=statistics.median(s["value"] for s in samples))
    value = base["value"]
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
                   "timing": "each step a 2^24-element sample of the workload; ms_per_step "
                             "extrapolated to its 8,030,261,248 parameters"},
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
    elif args.workload == "nvlink-exchange":
        run_nvlink_exchange(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
