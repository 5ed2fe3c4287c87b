"""The BASELINE configurations at their own shapes on the GPU, every byte against
the CPU oracle:

* config 3: momentum SGD over the 148 GPT-2-small tensors (124,439,808 FP32
  parameters), BF16 stochastic momentum, lr 1e-2, momentum 0.9, seed 11,
  gradients ~N(0, 1e-3) drawn afresh every step, 100 steps; parameters and
  states compared after every step (benchmarks/bench_optimizer_steps.py:33-53
  gives the shapes);
* config 5: AdamW at the Llama-3-70B shape, reduced to one decoder layer
  (855,654,400 parameters) and the final RMSNorm, two groups (vectors:
  weight decay 0, AdamW step 5; matrices: weight decay 0.1, AdamW step 6), BF16
  parameters and gradients ~N(0, 1e-4), FP16 stochastic moments, seed 3;
  two steps, every byte;
* config 2: the standalone cast of 2^24- and 2^26-element FP32 tensors
  (magnitudes 2^U(-20, 18), random signs, 1% specials) into BF16, FP16, E4M3
  and E5M2 under both rules, seed 7, the offset advanced by numel between
  casts, checked in 2^24-element chunks (benchmarks/cast_checks.py:10-67 gives
  the special-value families).

Tolerance: exact, except that a NaN only has to be NaN (the reference's policy).
"""

import math

import numpy as np
import pytest
import torch

import oracle
from _support import FMT, assert_bits_or_nan, tbits

pytestmark = pytest.mark.gpu

THREADS = oracle.cpu_threads()


def _threads(n):
    return THREADS if n >= 1 << 20 else 1


# ----------------------------------------------------------- config 3 ------

def test_config3_sgdm_gpt2_small_100_steps_every_byte(cuda_device):
    from sr_states.shapes import gpt2_small

    shapes = [s for _, s in gpt2_small()]
    assert len(shapes) == 148 and sum(math.prod(s) for s in shapes) == 124_439_808
    run_config3(shapes, 100, cuda_device)


def run_config3(shapes, steps, cuda_device):
    from sr_states import SGDMReferenceSR, StateFormat

    gen = torch.Generator(device=cuda_device).manual_seed(11)
    params = [torch.nn.Parameter(torch.empty(s, device=cuda_device).normal_(0, 0.02,
                                                                           generator=gen))
              for s in shapes]
    opt = SGDMReferenceSR(params, lr=1e-2, momentum=0.9, seed=11,
                          state_format={"momentum_buffer": StateFormat(torch.bfloat16,
                                                                       "stochastic")})
    host_p = [tbits(p).view(np.float32).reshape(-1).copy() for p in params]
    host_u = [np.zeros(p.numel(), np.uint16) for p in params]
    for step in range(1, steps + 1):
        for p in params:
            p.grad = torch.empty_like(p).normal_(0, 1e-3, generator=gen)
        opt.step()
        for i, p in enumerate(params):
            g = tbits(p.grad).view(np.float32).reshape(-1)
            oracle.sgdm_(host_p[i], g, host_u[i], u_fmt=oracle.BF16, u_rule=oracle.STOCHASTIC,
                         lr=1e-2, momentum=0.9, update_key=oracle.update_key(11, step, i),
                         threads=_threads(p.numel()))
            assert np.array_equal(tbits(p).reshape(-1), host_p[i].view(np.uint32)), (step, i)
            u = tbits(opt.state[p]["momentum_buffer"]).reshape(-1)
            assert np.array_equal(u, host_u[i]), (step, i)


# ----------------------------------------------------------- config 5 ------

def test_config5_adamw_llama3_70b_layer_two_groups_fp16_states(cuda_device):
    from sr_states.shapes import _llama

    named = [(n, s) for n, s in _llama(1, 8192, 8 * 128, 28672) if n not in ("embed_tokens",
                                                                             "lm_head")]
    assert sum(math.prod(s) for _, s in named if len(s) == 2) == 855_638_016
    run_config5(named, cuda_device)


def run_config5(named, cuda_device):
    from sr_states import AdamWReferenceSR, StateFormat

    vectors = [s for _, s in named if len(s) == 1]
    matrices = [s for _, s in named if len(s) == 2]
    gen = torch.Generator(device=cuda_device).manual_seed(3)

    def bf16(shape, std):
        return torch.empty(shape, device=cuda_device).normal_(0, std, generator=gen).to(
            torch.bfloat16)

    params = [torch.nn.Parameter(bf16(s, 0.02)) for s in vectors + matrices]
    fmt = {"exp_avg": StateFormat(torch.float16, "stochastic"),
           "exp_avg_sq": StateFormat(torch.float16, "stochastic")}
    n_vec = len(vectors)
    opt = AdamWReferenceSR([{"params": params[:n_vec], "weight_decay": 0.0},
                            {"params": params[n_vec:], "weight_decay": 0.1}],
                           lr=3e-4, betas=(0.9, 0.999), eps=1e-8, state_format=fmt, seed=3)
    # Existing moments at AdamW steps 4 and 5, so the next steps are 5 and 6.
    for i, p in enumerate(params):
        opt.state[p]["step"] = 4 if i < n_vec else 5
        opt.state[p]["exp_avg"] = bf16(p.shape, 1e-4).to(torch.float16)
        opt.state[p]["exp_avg_sq"] = bf16(p.shape, 1e-4).float().square().to(torch.float16)
    host = [{"p": tbits(p).reshape(-1).copy(),
             "m": tbits(opt.state[p]["exp_avg"]).reshape(-1).copy(),
             "v": tbits(opt.state[p]["exp_avg_sq"]).reshape(-1).copy()} for p in params]
    for rng_step in (1, 2):
        for p in params:
            p.grad = bf16(p.shape, 1e-4)
        opt.step()
        for i, p in enumerate(params):
            h = host[i]
            adam_step = (4 if i < n_vec else 5) + rng_step
            oracle.adamw_(h["p"], tbits(p.grad).reshape(-1).copy(), h["m"], h["v"],
                          m_fmt=oracle.F16, m_rule=oracle.STOCHASTIC, v_fmt=oracle.F16,
                          v_rule=oracle.STOCHASTIC, lr=3e-4, beta1=0.9, beta2=0.999, eps=1e-8,
                          weight_decay=0.0 if i < n_vec else 0.1, step=adam_step,
                          update_key=oracle.update_key(3, rng_step, i),
                          threads=_threads(p.numel()))
            context = f"step {rng_step} param {i}"
            assert np.array_equal(tbits(p).reshape(-1), h["p"]), context
            assert_bits_or_nan(tbits(opt.state[p]["exp_avg"]), h["m"], oracle.F16, context)
            assert_bits_or_nan(tbits(opt.state[p]["exp_avg_sq"]), h["v"], oracle.F16, context)
            assert opt.state[p]["step"] == adam_step


# ----------------------------------------------------------- config 2 ------

# FP32 encodings of the special values: +-0, +-Inf, NaN (quiet and signalling,
# both signs), FP32 subnormals, and per target format the value just above its
# largest finite one and the midpoint between that and the next grid step.
SPECIALS = np.array([
    0x00000000, 0x80000000, 0x7F800000, 0xFF800000, 0x7FC00000, 0xFFC00000, 0x7F800001,
    0x00000001, 0x80000001, 0x007FFFFF, 0x00400000, 0x80123456,
    0x7F7F0001, 0x7F7F8000, 0xFF7F8000,          # BF16 max 0x7F7F: next, midpoint above
    0x477FE001, 0x47800000, 0xC77FF000, 0x477FF000,  # FP16 max 65504
    0x43E00001, 0x43F00000, 0xC3F00000,          # E4M3 max 448: next, 480
    0x47600001, 0x47700000, 0xC7700000,          # E5M2 max 57344: next, 61440
], dtype=np.uint32)


def _sweep_input(n, seed):
    rng = np.random.default_rng(seed)
    x = np.exp2(rng.uniform(-20, 18, n)).astype(np.float32)
    x *= np.where(rng.random(n) < 0.5, -1, 1).astype(np.float32)
    bits = x.view(np.uint32)
    where = rng.integers(0, n, n // 100)
    bits[where] = SPECIALS[rng.integers(0, SPECIALS.size, where.size)]
    return x


@pytest.mark.parametrize("n", [1 << 24, 1 << 26], ids=["2^24", "2^26"])
def test_config2_cast_sweep_in_chunks(n, cuda_device):
    from sr_states import cast

    x = _sweep_input(n, 7 + n.bit_length())
    xd = torch.from_numpy(x).to(cuda_device)
    chunk = 1 << 24
    offset = 0
    for dtype in (torch.bfloat16, torch.float16, torch.float8_e4m3fn, torch.float8_e5m2):
        fmt = FMT[dtype]
        for rounding, rule in (("stochastic", oracle.STOCHASTIC), ("nearest", oracle.NEAREST)):
            y = tbits(cast(xd, dtype=dtype, rounding=rounding, seed=7, offset=offset))
            for lo in range(0, n, chunk):
                hi = min(n, lo + chunk)
                expected = oracle.cast(x[lo:hi], fmt, rule, seed=7, offset=offset + lo,
                                       threads=THREADS)
                assert_bits_or_nan(y[lo:hi], expected, fmt,
                                   f"{dtype} {rounding} chunk {lo // chunk}")
            offset += n  # advanced between repeated casts, as the reference's users do
