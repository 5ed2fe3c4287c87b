"""Replay the reference optimizer scenarios of tests/golden/optimizers.* through
this package's optimizer classes and compare every step with the reference bytes.

Parameters are teacher-forced: after each step's comparison the parameter is
reset to the reference's bytes, so a one-ulp difference (PyTorch's CPU sqrt is
not correctly rounded) never compounds.  States never depend on parameters.
AdamW parameters are checked with the reference's own intermediates of each
update (tests/golden/optimizers_intermediates.npz): equal to its update formula
evaluated with a correctly rounded square root, byte for byte.
"""

from __future__ import annotations

import numpy as np
import torch

import oracle
from _support import (FMT, assert_bits_or_nan, explain_adamw_param, from_bits, load_json,
                      load_npz, tbits, ulp_distance)


def scenarios():
    return load_json("optimizers.json")["scenarios"]


def _classes():
    import sr_states

    return {"adamw": sr_states.AdamWReferenceSR, "sgdm": sr_states.SGDMReferenceSR}


def build(spec, arrays, device, cls=None):
    from sr_states import StateFormat

    name, names = spec["name"], spec["state_names"]
    shapes = [(tuple(s), getattr(torch, d)) for s, d in spec["shapes"]]
    params = [torch.nn.Parameter(from_bits(arrays[f"{name}__p{i}__init"], dt, device).reshape(s))
              for i, (s, dt) in enumerate(shapes)]
    groups = []
    for g in spec["groups"]:
        fmt = {n: StateFormat(getattr(torch, d), r) for n, (d, r) in zip(names, g["formats"])}
        hp = dict(g["hp"])
        if "betas" in hp:
            hp["betas"] = tuple(hp["betas"])
        groups.append({"params": [params[i] for i in g["params"]], "state_format": fmt,
                       "sr_seed": g["sr_seed"], **hp})
    cls = cls or _classes()[spec["kind"]]
    opt = cls(groups, lr=0.01) if spec["kind"] == "sgdm" else cls(groups)
    for tg, g in zip(opt.param_groups, spec["groups"]):
        tg["sr_step"] = g["sr_step"]
    for pid, init in spec["initial"].items():
        p = params[int(pid)]
        group = next(tg for tg in opt.param_groups if any(q is p for q in tg["params"]))
        for n, fmt in zip(names, opt._formats(group)):
            opt.state[p][n] = from_bits(arrays[f"{name}__p{pid}__{n}__init"], fmt.dtype,
                                        device).reshape(p.shape)
        opt.state[p]["step"] = init["step"]
    return params, opt


def replay(spec, device, cls=None, arrays=None):
    """Run the scenario; returns (total parameter elements compared, mismatching ones)."""
    arrays = arrays if arrays is not None else load_npz("optimizers.npz")
    intermediates = load_npz("optimizers_intermediates.npz")
    name, names, kind = spec["name"], spec["state_names"], spec["kind"]
    params, opt = build(spec, arrays, device, cls)
    skip = {tuple(x) for x in spec["grad_none"]}
    compared = mismatched = 0
    group_of = {i: g for g in spec["groups"] for i in g["params"]}
    for step in range(1, spec["steps"] + 1):
        previous = [tbits(p).reshape(-1).copy() for p in params]
        for i, p in enumerate(params):
            p.grad = None if (step, i) in skip else from_bits(
                arrays[f"{name}__p{i}__grad{step}"], p.dtype, device).reshape(p.shape)
        opt.step()
        for i, p in enumerate(params):
            context = f"{name} step {step} param {i}"
            golden = arrays[f"{name}__p{i}__step{step}"].reshape(-1)
            actual = tbits(p).reshape(-1)
            width = 8 * p.element_size()
            distance = ulp_distance(actual, golden, width)
            if kind == "sgdm":
                assert distance.max(initial=0) == 0, context
            elif f"{name}__p{i}__sqrt{step}" in intermediates:
                hp = group_of[i]["hp"]
                prev = (previous[i].view(np.float32) if width == 32
                        else (previous[i].astype(np.uint32) << 16).view(np.float32))
                beta1, beta2 = hp.get("betas", (0.9, 0.999))
                adam_step = int(arrays[f"{name}__p{i}__adamstep{step}"][0])
                scalars = oracle.adamw_scalars(hp["lr"], beta1, beta2, hp.get("eps", 1e-8),
                                               hp.get("weight_decay", 1e-2), adam_step)
                inter = [intermediates[f"{name}__p{i}__{k}{step}"].view(np.float32)
                         for k in ("v32", "sqrt", "m32")]
                explain_adamw_param(actual, golden, prev, *inter, scalars, width)
            else:  # no update this step (no gradient): unchanged
                assert distance.max(initial=0) == 0, context
            compared += distance.size
            mismatched += int(np.count_nonzero(distance))
            for n in names:
                key = f"{name}__p{i}__{n}__step{step}"
                if key in arrays:
                    st = opt.state[p][n]
                    assert_bits_or_nan(tbits(st), arrays[key], FMT[st.dtype], f"{context} {n}")
                else:
                    assert n not in opt.state[p], context
            if f"{name}__p{i}__adamstep{step}" in arrays:
                assert opt.state[p]["step"] == int(arrays[f"{name}__p{i}__adamstep{step}"][0])
            with torch.no_grad():  # teacher forcing
                p.copy_(from_bits(golden, p.dtype, device).reshape(p.shape))
    assert [g["sr_step"] for g in opt.param_groups] == spec["final_sr_step"]
    return compared, mismatched


# --------------------------------------------------------------------------
# The reference's own optimizer regression scenario (tests/golden/regression.*,
# recorded from the reference's scripts/record_optimizer_golden.py setup): three
# parameters of 17, 9 and 5 elements in two groups (lr 0.01 and 0.03), FP32 or
# BF16-nearest states, seed 2^32-13, seven steps whose gradients are
# sin(0.137 * index + step + i), missing when (step + i) % 4 == 0.  Not teacher
# forced: every byte after the seventh step must equal the reference's.

def regression_cases():
    return load_json("regression.json")["cases"]


def replay_regression(case, device):
    """Run one regression case on ``device``; returns the list of mismatches."""
    import sr_states

    cls = getattr(sr_states, case["class"])
    pdtype = getattr(torch, case["param_dtype"].split(".")[-1])
    state_dtype = getattr(torch, case["state_dtype"].split(".")[-1])
    arrays = load_npz("regression.npz")
    params = [torch.nn.Parameter(torch.linspace(-1, 1, n).to(device, pdtype))
              for n in (17, 9, 5)]
    opt = cls([{"params": params[:2]}, {"params": params[2:], "lr": 0.03}], lr=0.01,
              state_dtype=state_dtype, rounding="nearest", seed=2**32 - 13)
    for step in range(7):
        for i, p in enumerate(params):
            p.grad = (None if (step + i) % 4 == 0 else
                      torch.sin(torch.arange(p.numel()).float() * 0.137 + step + i)
                      .to(device, pdtype))
        opt.step()
    bad, key = [], case["key"]
    for i, p in enumerate(params):
        if not np.array_equal(tbits(p), arrays[f"{key}/param{i}"]):
            bad.append(f"param{i}")
        for name in opt._state_names:
            if not np.array_equal(tbits(opt.state[p][name]), arrays[f"{key}/param{i}/{name}"]):
                bad.append(f"param{i}/{name}")
        if str(i) in case["steps"] and opt.state[p].get("step") != case["steps"][str(i)]:
            bad.append(f"param{i}/step")
    return bad
