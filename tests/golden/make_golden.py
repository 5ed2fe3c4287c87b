"""Generate the golden vectors of tests/golden/ by running the reference itself.

    python tests/golden/make_golden.py --reference /path/to/stochastic-rounding-pytorch
    (or set SR_STATES_REFERENCE to that path)

Imports the reference package ``sr_states`` (KristiTopollai/stochastic-rounding-pytorch,
pure Python on PyTorch's CPU kernels) from the given checkout and records its
outputs on seeded synthetic inputs:

  keys.json        update_key / state_key known answers (incl. the reference's own KATs)
  casts.npz        sr_states.cast outputs for the reference's cast test families and the
                   BASELINE config-2 synthetic sweep (input bits + output bits)
  functional.npz   adamw_step_ / sgdm_step_ on one tensor at offset 2^32-211
  config1.npz      BASELINE config 1 (AdamW, FP32 param, BF16 SR states, 10 steps) at
                   n = 2^13, every step's bytes
  config1_intermediates.npz  the reference's own v32, v32.sqrt() and m32 of every step
                   of that run (where its CPU sqrt is not correctly rounded)
  optimizers_intermediates.npz  the same intermediates for every AdamW update of
                   the optimizer scenarios below
  config1_full.json  the same run at n = 2^20: SHA-256 of the state bytes after each step
  optimizers.npz / optimizers.json
                   multi-parameter, multi-group optimizer scenarios (param_index, RNG
                   step, skipped gradients, AdamW bias-correction steps, mixed formats)

  regression.npz / regression.json
                   the scenario of the reference's own optimizer regression fixture
                   (scripts/record_optimizer_golden.py, checked by
                   tests/test_state_formats.py:44-100): AdamW and SGDM, FP32 and BF16
                   parameters, FP32 and BF16-nearest states, 3 parameters in 2 groups,
                   missing gradients, seed 2^32-13, 7 steps.  Recorded by running the
                   reference here, as that test re-derives its bytes in the current
                   environment (its committed capture is from macOS/ARM and differs on
                   x86 for the reference itself).

Only this script touches the reference; tests read the files it wrote.  Must be
run with the reference (not this repository's sr_states) importable.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

FMT_CODE = {"float32": 0, "bfloat16": 1, "float16": 2, "float8_e4m3fn": 3, "float8_e5m2": 4}


def bits(t):
    import torch

    width = {4: (torch.int32, np.uint32), 2: (torch.int16, np.uint16), 1: (torch.uint8, np.uint8)}
    tv, nv = width[t.dtype.itemsize]
    return t.detach().contiguous().view(tv).numpy().view(nv).copy()


def from_bits(a, dtype):
    import torch

    width = {4: torch.int32, 2: torch.int16, 1: torch.uint8}[dtype.itemsize]
    signed = {4: np.int32, 2: np.int16, 1: np.uint8}[dtype.itemsize]
    return torch.from_numpy(np.ascontiguousarray(a).view(signed).copy()).view(width).view(dtype)


def dtype_name(dt) -> str:
    return str(dt).replace("torch.", "")


# ------------------------------------------------------------------- keys --

def make_keys(ref):
    from sr_states._hash import state_key, update_key

    rng = np.random.default_rng(20260)
    triples = [
        (0, 0, 0), (0, 1, 0), (42, 17, 9),
        (0x12345678ABCDEFFE, 0xFEDCBA9876543210, 0xA5A5A5A5), (-1, 1 << 32, 1),
        (1, 16, 0), (-1, 2**32 + 1, 2**32 - 1), (2**87 + 7, 2**64 + 2**63 + 16, 2**39 + 13),
        (-(2**48) + 15, 2**32 - 1, 2**31 + 1), (0xFEDCBA9876543210, 2**32 + 1, 1),
    ]
    for _ in range(500):
        seed = int(rng.integers(-(2**62), 2**62)) * int(rng.integers(1, 4))
        step = int(rng.integers(0, 2**63)) >> int(rng.integers(0, 60))
        index = int(rng.integers(0, 2**32))
        triples.append((seed, step, index))
    update = [[s, t, i, update_key(s, t, i)] for s, t, i in triples]
    state_pairs = [(0, 0), (0, 1), (1, 0), (0x89ABCDEF, 1), (0xFFFFFFFF, 2)]
    state_pairs += [(int(k), int(j)) for k, j in zip(rng.integers(0, 2**32, 200),
                                                        rng.integers(0, 3, 200))]
    state = [[k, j, state_key(k, j)] for k, j in state_pairs]
    counters = rng.integers(0, 2**32, 4096, dtype=np.uint64)
    import torch
    from sr_states._hash import _u32_hash

    hashed = _u32_hash(torch.from_numpy(counters.astype(np.int64)), 0).numpy()
    return {"update_key": update, "state_key": state,
            "h32": {"counters": counters.tolist(), "hashes": hashed.astype(np.uint64).tolist()}}


# ------------------------------------------------------------------ casts --

def _cast_check_families():
    """Input families of the reference's BF16 cast checks (benchmarks/cast_checks.py:10-67)."""
    import torch

    gen = torch.Generator().manual_seed(91)
    out = []
    for n in (1, 127, 128, 129, 255, 257, 513, 4097, 100_003):
        b = torch.randint(0, 2**32, (n,), generator=gen, dtype=torch.int64)
        out.append((f"cc_random_{n}", b.to(torch.int32).view(torch.float32), 7, 2**32 - 13))
    exact = (torch.arange(65536, dtype=torch.int64) << 16).to(torch.int32)
    out.append(("cc_exact_bf16", exact.view(torch.float32), 0, 0))
    boundaries = torch.tensor(
        [0, 1, 0x7FFF, 0x8000, 0xFFFF, 0x10000, 0x7FFFFF, 0x800000, 0x3F807FFF, 0x3F808000,
         0x3F808001, 0x7F7FFFFF, 0x7F800000, 0x7F800001, 0x7FC00000], dtype=torch.int64)
    b = torch.cat((boundaries, boundaries | 0x80000000)).to(torch.int32)
    for k, (seed, offset) in enumerate(((2**32 + 9, -17), (991, 2**32 - 31))):
        out.append((f"cc_boundary_{k}", b.view(torch.float32).repeat(19), seed, offset))
    return out


def _positive_grid(dtype):
    import torch

    if dtype == torch.float16:
        values = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(dtype).float()
    else:
        values = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(dtype).float()
    return values[torch.isfinite(values) & ~torch.signbit(values)].sort().values


def _boundary_inputs(dtype):
    """Grid points, midpoints and their FP32 neighbours (tests/test_minifloat.py:27-52)."""
    import torch

    grid = _positive_grid(dtype)
    mid = (grid[:-1] + grid[1:]) * 0.5
    up = torch.nextafter(mid, torch.full_like(mid, float("inf")))
    down = torch.nextafter(mid, torch.zeros_like(mid))
    mx = float(torch.finfo(dtype).max)
    extra = torch.tensor([mx, mx + 16, 2.0**-149, 2.0**-126, 1e-30, 1e30, float("inf"),
                          float("nan")])
    positive = torch.cat((grid, mid, up, down, extra))
    return torch.cat((positive, -positive))


def _config2_inputs(n, dtype_list, gen):
    """log-uniform magnitudes in [2^-20, 2^18], random sign, 1% specials."""
    import torch

    mag = torch.exp2(torch.rand(n, generator=gen, dtype=torch.float64) * 38.0 - 20.0)
    sign = torch.where(torch.rand(n, generator=gen) < 0.5, -1.0, 1.0).double()
    x = (mag * sign).float()
    specials = [0.0, -0.0, float("inf"), float("-inf"), float("nan"), 1e-40, -1e-40, 2.0**-149]
    for dt in dtype_list:
        mx = torch.tensor(float(torch.finfo(dt).max))
        above = torch.nextafter(mx, torch.tensor(float("inf"))).item()
        grid = _positive_grid(dt)
        half_step = (grid[-1] - grid[-2]).item() / 2
        specials += [above, -above, mx.item() + half_step, -(mx.item() + half_step)]
    count = n // 100
    where = torch.randperm(n, generator=gen)[:count]
    pick = torch.randint(0, len(specials), (count,), generator=gen)
    x[where] = torch.tensor(specials, dtype=torch.float32)[pick]
    return x


def make_casts(ref):
    import torch

    cast = ref.cast
    arrays = {}
    manifest = []

    def record(name, x, dtype, rounding, seed, offset):
        y = cast(x, dtype=dtype, rounding=rounding, seed=seed, offset=offset)
        key = f"{name}__{dtype_name(dtype)}__{rounding}__{len(manifest)}"
        if f"{name}__x" not in arrays:
            arrays[f"{name}__x"] = bits(x.reshape(-1))
        arrays[key] = bits(y.reshape(-1))
        manifest.append({"key": key, "input": f"{name}__x", "format": FMT_CODE[dtype_name(dtype)],
                         "rule": 1 if rounding == "stochastic" else 0, "seed": seed,
                         "offset": offset})

    for name, x, seed, offset in _cast_check_families():
        record(name, x, torch.bfloat16, "stochastic", seed, offset)
        record(name, x, torch.bfloat16, "nearest", 0, 0)
    high = torch.arange(0x7F80, dtype=torch.int64) << 16
    mids = (high[:, None] + torch.tensor([0x7FFF, 0x8000, 0x8001])).flatten()
    mids = torch.cat((mids, mids | 0x80000000)).to(torch.int32).view(torch.float32)
    record("bf16_midpoints", mids, torch.bfloat16, "nearest", 0, 0)

    gen = torch.Generator().manual_seed(541)
    random_bits = torch.randint(-(2**31), 2**31, (10007,), generator=gen, dtype=torch.int32)
    for dt in (torch.float8_e4m3fn, torch.float8_e5m2, torch.float16):
        x = _boundary_inputs(dt)
        if dt == torch.float16:
            x = x[::5]
        x = torch.cat((x, random_bits.view(torch.float32)))
        name = f"minifloat_boundary_{dtype_name(dt)}"
        for rounding in ("nearest", "stochastic"):
            record(name, x, dt, rounding, 2**32 - 7, 2**32 - 93)

    gen = torch.Generator().manual_seed(7)
    formats = (torch.bfloat16, torch.float16, torch.float8_e4m3fn, torch.float8_e5m2)
    x = _config2_inputs(1 << 16, formats, gen)
    for dt in formats:
        for rounding in ("stochastic", "nearest"):
            for repeat in range(2):
                record("config2", x, dt, rounding, 7, repeat * x.numel())
    return arrays, manifest


# ------------------------------------------------------------- functional --

def make_functional(ref):
    """adamw_step_/sgdm_step_ on 1031 elements at offset 2^32-211 with dyadic gradients
    (tests/test_triton_states.py:37-64)."""
    import torch
    from sr_states._hash import update_key
    from sr_states.reference.adamw import adamw_step_
    from sr_states.reference.sgd import sgdm_step_

    arrays, manifest = {}, []
    g = 1.0 + torch.arange(1031, dtype=torch.float32) / 2048
    key = update_key(0xFEDCBA9876543210, (1 << 32) + 1, 7)
    offset = (1 << 32) - 211
    arrays["grad"] = bits(g)
    for kind in ("adamw", "sgdm"):
        for dt in (torch.bfloat16, torch.float16, torch.float8_e4m3fn, torch.float8_e5m2):
            for rounding in ("stochastic", "nearest"):
                states = [torch.zeros_like(g, dtype=dt) for _ in range(2 if kind == "adamw" else 1)]
                p = torch.linspace(-1, 1, g.numel())
                tensors = (p, g.clone(), *states)
                if kind == "adamw":
                    adamw_step_(*tensors, lr=0.01, beta1=0.5, beta2=0.5, eps=0.125,
                                weight_decay=0.0, step=1, state_dtype=dt, rounding=rounding,
                                seed=key, offset=offset)
                else:
                    sgdm_step_(*tensors, lr=0.01, momentum_factor=0.5, state_dtype=dt,
                               rounding=rounding, seed=key, offset=offset)
                name = f"{kind}__{dtype_name(dt)}__{rounding}"
                arrays[f"{name}__param"] = bits(tensors[0])
                for i, s in enumerate(tensors[2:]):
                    arrays[f"{name}__state{i}"] = bits(s)
                manifest.append({"name": name, "kind": kind, "format": FMT_CODE[dtype_name(dt)],
                                 "rule": 1 if rounding == "stochastic" else 0, "key": key,
                                 "offset": offset})
    return arrays, manifest


# ---------------------------------------------------------------- config1 --

def run_config1(ref, n, steps=10, record_all=True):
    """one FP32 parameter ~N(0, 0.02), FP32 gradient ~N(0, 1e-3)
    regenerated each step, BF16 SR states, lr=3e-4, betas=(0.9, 0.999), eps=1e-8,
    weight_decay=0.01, seed=7, 10 steps (AdamWReferenceSR)."""
    import torch

    gen = torch.Generator().manual_seed(1234)
    p = torch.nn.Parameter(torch.randn(n, generator=gen) * 0.02)
    opt = ref.AdamWReferenceSR([p], lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                               state_dtype=torch.bfloat16, rounding="stochastic", seed=7)
    arrays = {"param_init": bits(p)} if record_all else {}
    digests = []
    for step in range(1, steps + 1):
        p.grad = torch.randn(n, generator=gen) * 1e-3
        if record_all:
            arrays[f"grad_{step}"] = bits(p.grad)
        opt.step()
        st = opt.state[p]
        if record_all:
            arrays[f"param_{step}"] = bits(p)
            arrays[f"exp_avg_{step}"] = bits(st["exp_avg"])
            arrays[f"exp_avg_sq_{step}"] = bits(st["exp_avg_sq"])
        digests.append({
            "step": step,
            "grad_sha256": hashlib.sha256(bits(p.grad).tobytes()).hexdigest(),
            "exp_avg_sha256": hashlib.sha256(bits(st["exp_avg"]).tobytes()).hexdigest(),
            "exp_avg_sq_sha256": hashlib.sha256(bits(st["exp_avg_sq"]).tobytes()).hexdigest(),
        })
    return arrays, digests


class _SqrtRecorder:
    """Records the FP32 intermediates of the reference's AdamW update while active:
    the input and output of its square root (``v32.sqrt()``,
    sr_states/reference/adamw.py:86) and the first moment m32 it passes to
    ``addcdiv_`` (:88)."""

    def __init__(self):
        import torch

        self.seen = {}
        self._torch = torch
        self._saved = None

    def __enter__(self):
        torch = self._torch
        real_sqrt, real_addcdiv = torch.Tensor.sqrt, torch.Tensor.addcdiv_
        seen = self.seen

        def sqrt(tensor):
            out = real_sqrt(tensor)
            seen["v32"], seen["sqrt"] = tensor.detach().clone(), out.detach().clone()
            return out

        def addcdiv_(tensor, tensor1, tensor2, *args, **kwargs):
            seen["m32"] = tensor1.detach().clone()
            return real_addcdiv(tensor, tensor1, tensor2, *args, **kwargs)

        self._saved = (real_sqrt, real_addcdiv)
        torch.Tensor.sqrt, torch.Tensor.addcdiv_ = sqrt, addcdiv_
        return self

    def __exit__(self, *exc):
        self._torch.Tensor.sqrt, self._torch.Tensor.addcdiv_ = self._saved
        return False


def record_adamw_intermediates(opt, params, sink):
    """Wrap ``opt._step_parameter`` so that each parameter update stores the
    reference's intermediates in ``sink[param index]`` (a fresh dict per update)."""
    original = opt._step_parameter
    index = {id(p): i for i, p in enumerate(params)}

    def step_parameter(parameter, *args, **kwargs):
        with _SqrtRecorder() as recorder:
            original(parameter, *args, **kwargs)
        sink[index[id(parameter)]] = dict(recorder.seen)

    opt._step_parameter = step_parameter


def run_config1_intermediates(ref, n, steps=10):
    """The same run as run_config1, recording the reference's own FP32
    intermediates of every step (see _SqrtRecorder).  PyTorch's CPU sqrt is not
    correctly rounded, and these bytes show exactly where it differs."""
    import torch

    gen = torch.Generator().manual_seed(1234)
    p = torch.nn.Parameter(torch.randn(n, generator=gen) * 0.02)
    opt = ref.AdamWReferenceSR([p], lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                               state_dtype=torch.bfloat16, rounding="stochastic", seed=7)
    arrays, sink = {}, {}
    record_adamw_intermediates(opt, [p], sink)
    for step in range(1, steps + 1):
        p.grad = torch.randn(n, generator=gen) * 1e-3
        sink.clear()
        opt.step()
        for name in ("v32", "sqrt", "m32"):
            arrays[f"{name}_{step}"] = bits(sink[0][name])
    return arrays


# ------------------------------------------------------------- optimizers --

def _scenario(ref, name, kind, groups, shapes, steps, grad_none=(), initial=None, init_seed=0,
              grad_scale=1e-3, init_scale=0.02):
    """Run one reference optimizer scenario and record every step's bytes.

    groups: list of dicts {params: [ids], hp: {...}, sr_seed, sr_step, formats: [[dtype, rule]]}
    shapes: list of (shape, param_dtype)
    initial: optional {param_id: {"step": int, "state_scale": float}} pre-existing AdamW state
    """
    import torch

    names = ("exp_avg", "exp_avg_sq") if kind == "adamw" else ("momentum_buffer",)
    cls = ref.AdamWReferenceSR if kind == "adamw" else ref.SGDMReferenceSR
    gen = torch.Generator().manual_seed(init_seed)
    params = [torch.nn.Parameter((torch.randn(s, generator=gen) * init_scale).to(dt))
              for s, dt in shapes]
    arrays = {}
    for i, p in enumerate(params):
        arrays[f"{name}__p{i}__init"] = bits(p)
    torch_groups = []
    for g in groups:
        fmt = {n: ref.StateFormat(getattr(torch, d), r) for n, (d, r) in zip(names, g["formats"])}
        torch_groups.append({"params": [params[i] for i in g["params"]], "state_format": fmt,
                             "sr_seed": g["sr_seed"], **g["hp"]})
    defaults = {"lr": 0.01} if kind == "sgdm" else {}
    opt = cls(torch_groups, **defaults)
    for tg, g in zip(opt.param_groups, groups):
        tg["sr_step"] = g["sr_step"]
    for pid, spec in (initial or {}).items():
        p = params[pid]
        fmts = opt._formats(next(tg for tg in opt.param_groups if any(q is p for q in tg["params"])))
        st = opt.state[p]
        for n, f in zip(names, fmts):
            init = (torch.randn(p.shape, generator=gen) * spec["state_scale"])
            if n == "exp_avg_sq":
                init = init.abs()
            st[n] = init.to(f.dtype)
            arrays[f"{name}__p{pid}__{n}__init"] = bits(st[n])
        st["step"] = spec["step"]
    skip = {tuple(x) for x in grad_none}
    sink = {}
    if kind == "adamw":
        record_adamw_intermediates(opt, params, sink)
    for step in range(1, steps + 1):
        for i, p in enumerate(params):
            if (step, i) in skip:
                p.grad = None
            else:
                p.grad = (torch.randn(p.shape, generator=gen) * grad_scale).to(p.dtype)
                arrays[f"{name}__p{i}__grad{step}"] = bits(p.grad)
        sink.clear()
        opt.step()
        for i, seen in sink.items():
            for key in ("v32", "sqrt", "m32"):
                arrays[f"{name}__p{i}__{key}{step}"] = bits(seen[key])
        for i, p in enumerate(params):
            arrays[f"{name}__p{i}__step{step}"] = bits(p)
            for n in names:
                if n in opt.state[p]:
                    arrays[f"{name}__p{i}__{n}__step{step}"] = bits(opt.state[p][n])
            if kind == "adamw" and "step" in opt.state[p]:
                arrays[f"{name}__p{i}__adamstep{step}"] = np.array([opt.state[p]["step"]])
    spec = {"name": name, "kind": kind, "state_names": list(names), "steps": steps,
            "shapes": [[list(s), dtype_name(dt)] for s, dt in shapes], "groups": groups,
            "grad_none": [list(x) for x in grad_none],
            "initial": {str(k): v for k, v in (initial or {}).items()},
            "final_sr_step": [tg["sr_step"] for tg in opt.param_groups]}
    return arrays, spec


def make_optimizers(ref):
    import torch

    bf, f32 = torch.bfloat16, torch.float32
    arrays, specs = {}, []

    def add(result):
        a, s = result
        arrays.update(a)
        specs.append(s)

    d, h = 32, 32 * 3
    gpt2 = [((131, d), f32), ((48, d), f32)]
    for _ in range(2):
        gpt2 += [((d,), f32), ((d,), f32), ((d, h), f32), ((h,), f32), ((d, d), f32), ((d,), f32),
                 ((d,), f32), ((d,), f32), ((d, 4 * d), f32), ((4 * d,), f32), ((4 * d, d), f32),
                 ((d,), f32)]
    gpt2 += [((d,), f32), ((d,), f32)]
    add(_scenario(ref, "sgdm_gpt2_like", "sgdm",
                  [{"params": list(range(len(gpt2))), "hp": {"lr": 1e-2, "momentum": 0.9},
                    "sr_seed": 11, "sr_step": 0, "formats": [["bfloat16", "stochastic"]]}],
                  gpt2, steps=4, grad_none=[(2, 3), (3, 0)], init_seed=1))

    llama = [((128, d), bf)]
    for _ in range(2):
        llama += [((d,), bf), ((d, d), bf), ((8, d), bf), ((8, d), bf), ((d, d), bf), ((d,), bf),
                  ((88, d), bf), ((88, d), bf), ((d, 88), bf)]
    llama += [((d,), bf), ((128, d), bf)]
    add(_scenario(ref, "adamw_llama_like_fp8", "adamw",
                  [{"params": list(range(len(llama))),
                    "hp": {"lr": 3e-4, "betas": (0.9, 0.999), "eps": 1e-8, "weight_decay": 0.1},
                    "sr_seed": 7, "sr_step": 0,
                    "formats": [["float8_e4m3fn", "stochastic"], ["bfloat16", "stochastic"]]}],
                  llama, steps=3, init_seed=2, grad_scale=1e-4))

    vectors = [i for i, (s, _) in enumerate(llama) if len(s) == 1]
    matrices = [i for i, (s, _) in enumerate(llama) if len(s) == 2]
    hp = {"lr": 3e-4, "betas": (0.9, 0.999), "eps": 1e-8}
    initial = {i: {"step": 4, "state_scale": 1e-4} for i in vectors}
    initial.update({i: {"step": 5, "state_scale": 1e-4} for i in matrices})
    add(_scenario(ref, "adamw_two_groups_fp16", "adamw",
                  [{"params": vectors, "hp": {**hp, "weight_decay": 0.0}, "sr_seed": 3,
                    "sr_step": 1000, "formats": [["float16", "stochastic"]] * 2},
                   {"params": matrices, "hp": {**hp, "weight_decay": 0.1}, "sr_seed": 3,
                    "sr_step": 1000, "formats": [["float16", "stochastic"]] * 2}],
                  llama, steps=2, initial=initial, init_seed=3, grad_scale=1e-4))

    mixed = [((37, 5), f32), ((129,), bf), ((1000,), f32), ((3,), bf), ((2049,), f32)]
    add(_scenario(ref, "adamw_mixed_rules", "adamw",
                  [{"params": [0, 1, 2],
                    "hp": {"lr": 1e-3, "betas": (0.8, 0.95), "eps": 1e-6, "weight_decay": 0.05},
                    "sr_seed": 2**64 - 5, "sr_step": 2**32 - 2,
                    "formats": [["float8_e4m3fn", "nearest"], ["float8_e5m2", "stochastic"]]},
                   {"params": [3, 4],
                    "hp": {"lr": 2e-3, "betas": (0.9, 0.99), "eps": 1e-7, "weight_decay": 0.0},
                    "sr_seed": -12345, "sr_step": 2**32 - 2,
                    "formats": [["bfloat16", "nearest"], ["float16", "stochastic"]]}],
                  mixed, steps=3, grad_none=[(2, 1)], init_seed=4, grad_scale=0.3,
                  init_scale=1.0))
    add(_scenario(ref, "adamw_fp32_states", "adamw",
                  [{"params": [0, 1, 2, 3, 4],
                    "hp": {"lr": 1e-2, "betas": (0.9, 0.999), "eps": 1e-8, "weight_decay": 0.01},
                    "sr_seed": 5, "sr_step": 0,
                    "formats": [["float32", "stochastic"], ["float32", "nearest"]]}],
                  mixed, steps=3, init_seed=5, grad_scale=0.1))
    add(_scenario(ref, "sgdm_fp8_fp16", "sgdm",
                  [{"params": [0, 2, 4], "hp": {"lr": 0.1, "momentum": 0.5}, "sr_seed": 99,
                    "sr_step": 7, "formats": [["float8_e5m2", "stochastic"]]},
                   {"params": [1, 3], "hp": {"lr": 0.05, "momentum": 0.8}, "sr_seed": 98,
                    "sr_step": 7, "formats": [["float16", "nearest"]]}],
                  mixed, steps=3, init_seed=6, grad_scale=0.5, init_scale=1.0))

    # RNG-stream specification (tests/test_rng_streams.py:86-119): a skipped
    # parameter in group 0, the high step word, four state dtypes.
    one = [((3,), f32), ((1031,), f32)]
    for kind in ("adamw", "sgdm"):
        for dt in ("bfloat16", "float16", "float8_e4m3fn", "float8_e5m2"):
            hp = ({"lr": 0.01, "betas": (0.5, 0.5), "eps": 0.125, "weight_decay": 0.0}
                  if kind == "adamw" else {"lr": 0.01, "momentum": 0.9})
            n_states = 2 if kind == "adamw" else 1
            add(_scenario(ref, f"rng_spec_{kind}_{dt}", kind,
                          [{"params": [0], "hp": hp, "sr_seed": 0, "sr_step": 1 << 32,
                            "formats": [[dt, "stochastic"]] * n_states},
                           {"params": [1], "hp": hp, "sr_seed": 0xFEDCBA9876543210,
                            "sr_step": 1 << 32, "formats": [[dt, "stochastic"]] * n_states}],
                          one, steps=1, grad_none=[(1, 0)], init_seed=8, grad_scale=1.0))
    return arrays, specs


REGRESSION_SIZES = (17, 9, 5)


def regression_gradient(n, step, i, dtype):
    """Gradient of parameter i at step (None when (step + i) % 4 == 0) of the
    reference's regression scenario."""
    import torch

    if (step + i) % 4 == 0:
        return None
    return torch.sin(torch.arange(n).float() * 0.137 + step + i).to(dtype)


def make_regression(ref):
    """The reference's optimizer regression scenario, run on the reference here."""
    import torch

    arrays, cases = {}, []
    for cls_name in ("SGDMReferenceSR", "AdamWReferenceSR"):
        cls = getattr(ref, cls_name)
        for policy, state_dtype in (("fp32", torch.float32), ("bf16_rn", torch.bfloat16)):
            for pdtype in (torch.float32, torch.bfloat16):
                params = [torch.nn.Parameter(torch.linspace(-1, 1, n).to(pdtype))
                          for n in REGRESSION_SIZES]
                opt = cls([{"params": params[:2]}, {"params": params[2:], "lr": 0.03}],
                          lr=0.01, state_dtype=state_dtype, rounding="nearest",
                          seed=2**32 - 13)
                for step in range(7):
                    for i, p in enumerate(params):
                        p.grad = regression_gradient(p.numel(), step, i, pdtype)
                    opt.step()
                key = f"{cls_name}/{policy}/{str(pdtype).split('.')[-1]}"
                case = {"key": key, "class": cls_name, "state_dtype": str(state_dtype),
                        "param_dtype": str(pdtype), "steps": {}}
                for i, p in enumerate(params):
                    arrays[f"{key}/param{i}"] = bits(p)
                    for name, value in opt.state[p].items():
                        if isinstance(value, torch.Tensor):
                            arrays[f"{key}/param{i}/{name}"] = bits(value)
                        else:
                            case["steps"][str(i)] = value
                cases.append(case)
    return arrays, cases


def _is_intermediate(key: str) -> bool:
    tail = key.rsplit("__", 1)[-1]
    return tail.startswith(("v32", "sqrt", "m32"))


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference", default=os.environ.get("SR_STATES_REFERENCE"),
                        help="checkout of the reference (default: $SR_STATES_REFERENCE)")
    parser.add_argument("--only", choices=("regression", "intermediates"),
                        default=None, help="write one fixture family only")
    args = parser.parse_args()
    if not args.reference:
        parser.error("give --reference or set SR_STATES_REFERENCE")
    sys.path.insert(0, str(Path(args.reference).resolve()))
    import sr_states as ref
    import torch

    assert Path(ref.__file__).resolve().is_relative_to(Path(args.reference).resolve()), ref.__file__
    torch.set_num_threads(8)
    meta = {"generator": "tests/golden/make_golden.py", "torch": str(torch.__version__),
            "reference_version": getattr(ref, "__version__", "?")}

    if args.only == "intermediates":
        np.savez_compressed(HERE / "config1_intermediates.npz",
                            **run_config1_intermediates(ref, 1 << 13))
        arrays, _ = make_optimizers(ref)
        np.savez_compressed(HERE / "optimizers_intermediates.npz",
                            **{k: v for k, v in arrays.items() if _is_intermediate(k)})
        return
    arrays, cases = make_regression(ref)
    np.savez_compressed(HERE / "regression.npz", **arrays)
    (HERE / "regression.json").write_text(json.dumps({"meta": meta, "cases": cases}, indent=1))
    if args.only == "regression":
        return
    (HERE / "keys.json").write_text(json.dumps({"meta": meta, **make_keys(ref)}))
    arrays, manifest = make_casts(ref)
    np.savez_compressed(HERE / "casts.npz", **arrays)
    (HERE / "casts.json").write_text(json.dumps({"meta": meta, "cases": manifest}, indent=1))
    arrays, manifest = make_functional(ref)
    np.savez_compressed(HERE / "functional.npz", **arrays)
    (HERE / "functional.json").write_text(json.dumps({"meta": meta, "cases": manifest}, indent=1))
    arrays, _ = run_config1(ref, 1 << 13)
    np.savez_compressed(HERE / "config1.npz", **arrays)
    np.savez_compressed(HERE / "config1_intermediates.npz",
                        **run_config1_intermediates(ref, 1 << 13))
    _, digests = run_config1(ref, 1 << 20, record_all=False)
    (HERE / "config1_full.json").write_text(json.dumps(
        {"meta": meta, "n": 1 << 20, "seed_generator": 1234, "steps": digests}, indent=1))
    arrays, specs = make_optimizers(ref)
    intermediates = {k: arrays.pop(k) for k in list(arrays) if _is_intermediate(k)}
    np.savez_compressed(HERE / "optimizers_intermediates.npz", **intermediates)
    np.savez_compressed(HERE / "optimizers.npz", **arrays)
    (HERE / "optimizers.json").write_text(json.dumps({"meta": meta, "scenarios": specs},
                                                     indent=1))
    print("wrote", sorted(p.name for p in HERE.iterdir()))


if __name__ == "__main__":
    main()
