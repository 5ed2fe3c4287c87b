"""Drop-in API contracts on CPU (launches, where any, run the oracle stand-in):
formats, the rounding registry, validation messages, checkpoints and RNG keys."""

import copy

import pytest
import torch

import sr_states
import sr_states.rounding as rounding_module
from sr_states import (AdamWReferenceRN, AdamWReferenceSR, SGDMReferenceRN, SGDMReferenceSR,
                       StateFormat, StateOptimizer, cast, register_rounding)
from sr_states._hash import split_words, update_key
from sr_states.cuda import cuda_adamw_step_, cuda_sgdm_step_
from sr_states.rounding import validate_rounding
from sr_states.triton import AdamWTriton, SGDMTriton

CLASSES = [AdamWReferenceSR, SGDMReferenceSR, AdamWTriton, SGDMTriton]


@pytest.fixture(autouse=True)
def isolated_registry(monkeypatch):
    monkeypatch.setattr(rounding_module, "_RULES", rounding_module._RULES.copy())


def toward_zero(x, *, dtype, seed, offset):
    bits = x.contiguous().view(torch.int32) & -65536
    return bits.view(torch.float32).to(dtype)


def test_public_names():
    assert set(sr_states.__all__) == {"AdamWReferenceRN", "AdamWReferenceSR", "SGDMReferenceRN",
                                      "SGDMReferenceSR", "StateFormat", "StateOptimizer", "cast",
                                      "register_rounding"}
    import sr_states.triton as tri

    for name in ("AdamWTriton", "SGDMTriton", "cast", "is_triton_available", "rn_cast_bf16",
                 "sr_cast_bf16", "triton_adamw_step_", "triton_sgdm_step_"):
        assert hasattr(tri, name)
    assert issubclass(SGDMTriton, torch.optim.Optimizer)


def test_state_format_serialization_and_backends():
    fmt = StateFormat(torch.bfloat16, "nearest")
    assert StateFormat.from_dict(fmt.to_dict()) == fmt
    for backend in ("reference", "compiled", "cuda", "triton"):
        fmt.validate(backend)
    with pytest.raises(ValueError, match="backend"):
        fmt.validate("missing")
    for invalid in ({"dtype": torch.bfloat16},
                    {"dtype": torch.bfloat16, "rounding": "nearest", "extra": 1}):
        with pytest.raises(ValueError):
            StateFormat.from_dict(invalid)


@pytest.mark.parametrize("cls", CLASSES)
def test_format_validation_and_group_overrides(cls):
    p, q = [torch.nn.Parameter(torch.ones(3)) for _ in range(2)]
    fmt = StateFormat(torch.float32, "nearest")
    for extra in ({"state_dtype": torch.float32}, {"rounding": "nearest"}):
        with pytest.raises(ValueError, match="combined"):
            cls([p], lr=0.1, state_format=fmt, **extra)
    with pytest.raises(TypeError, match="StateFormat"):
        cls([{"params": [p], "state_format": (fmt,) * len(cls._state_names)}], lr=0.1)
    with pytest.raises(ValueError, match="keys"):
        cls([p], lr=0.1, state_format={"bad": fmt})
    opt = cls([{"params": [p], "state_format": fmt}], lr=0.1)
    assert all(f["dtype"] == torch.float32 for f in opt.param_groups[0]["state_format"].values())
    opt.add_param_group({"params": [q], "rounding": "nearest"})
    assert all(f == StateFormat(torch.bfloat16, "nearest").to_dict()
               for f in opt.param_groups[1]["state_format"].values())
    with pytest.raises(ValueError, match="registered"):
        opt.add_param_group({"params": [torch.nn.Parameter(torch.ones(1))],
                             "state_format": StateFormat(torch.bfloat16, "missing")})
    with pytest.raises(ValueError):
        opt.add_param_group({"params": [torch.nn.Parameter(torch.ones(1))], "lr": -1})
    assert len(opt.param_groups) == 2


def test_registry_validation():
    nearest = lambda x, **kw: x.to(kw["dtype"])  # noqa: E731
    with pytest.raises(ValueError, match="already registered"):
        register_rounding("nearest", torch.bfloat16, reference=nearest)
    with pytest.raises(ValueError, match="nonempty"):
        register_rounding("", torch.bfloat16, reference=nearest)
    with pytest.raises(ValueError, match="floating-point"):
        register_rounding("rule", torch.int32, reference=nearest)
    with pytest.raises(TypeError, match="callable"):
        register_rounding("rule", torch.bfloat16, reference=None)
    with pytest.raises(ValueError, match="native"):
        register_rounding("rule", torch.bfloat16, reference=nearest, native="round_up")
    with pytest.raises(ValueError, match="backend"):
        validate_rounding(torch.bfloat16, "nearest", backend="unknown")
    for dtype in (torch.float8_e4m3fn, torch.float8_e5m2, torch.float16):
        for mode in ("nearest", "stochastic"):
            with pytest.raises(ValueError, match="already registered"):
                register_rounding(mode, dtype, reference=nearest)


@pytest.mark.parametrize("cls", CLASSES)
def test_fused_optimizers_reject_rules_without_a_native_kernel(cls):
    register_rounding("toward_zero", torch.bfloat16, reference=toward_zero)
    # The Triton-named classes keep the reference's message
    # (tests/test_rounding_registry.py:85-89 of the reference).
    backend = "Triton" if cls in (AdamWTriton, SGDMTriton) else "CUDA"
    with pytest.raises(ValueError, match=f"no {backend} implementation"):
        cls([torch.nn.Parameter(torch.ones(1))], lr=0.1, rounding="toward_zero")
    with pytest.raises(ValueError, match="no Triton implementation"):
        validate_rounding(torch.bfloat16, "toward_zero", backend="triton")


def test_registered_rule_with_native_implementation_runs_fused(fake_launcher):
    register_rounding("my_sr", torch.bfloat16, reference=toward_zero, native="stochastic")
    p, q = torch.nn.Parameter(torch.ones(17)), torch.nn.Parameter(torch.ones(17))
    a = SGDMReferenceSR([p], lr=0.1, rounding="my_sr", seed=3)
    b = SGDMReferenceSR([q], lr=0.1, seed=3)
    p.grad = q.grad = torch.linspace(-1, 1, 17)
    a.step()
    b.step()
    assert torch.equal(a.state[p]["momentum_buffer"], b.state[q]["momentum_buffer"])
    assert a.param_groups[0]["state_format"]["momentum_buffer"]["rounding"] == "my_sr"


def test_cast_contract_and_custom_reference_rules():
    register_rounding("toward_zero", torch.bfloat16, reference=toward_zero)
    x = torch.tensor([1.003, -1.006, 0.0, -0.0])
    assert torch.equal(cast(x, dtype=torch.bfloat16, rounding="toward_zero"), toward_zero(
        x, dtype=torch.bfloat16, seed=0, offset=0))
    assert cast(x, dtype=torch.float32) is x or torch.equal(cast(x, dtype=torch.float32), x)
    with pytest.raises(TypeError, match="float32"):
        cast(x.double(), dtype=torch.bfloat16)
    register_rounding("bad_dtype", torch.bfloat16, reference=lambda x, **kw: x)
    register_rounding("bad_shape", torch.bfloat16, reference=lambda x, **kw: x[:1].bfloat16())
    register_rounding("not_tensor", torch.bfloat16, reference=lambda x, **kw: None)
    for name in ("bad_dtype", "bad_shape"):
        with pytest.raises(ValueError, match="requested dtype"):
            cast(torch.ones(2), dtype=torch.bfloat16, rounding=name)
    with pytest.raises(TypeError, match="return a tensor"):
        cast(torch.ones(2), dtype=torch.bfloat16, rounding="not_tensor")
    with pytest.raises(ValueError, match="CUDA"):
        cast(torch.ones(2), dtype=torch.bfloat16)  # built-ins run on the sm_100a kernel


def test_cast_runs_builtins_through_the_kernel_path(fake_launcher):
    import numpy as np

    import oracle

    x = torch.linspace(-3, 7, 35 * 9).reshape(35, 9).T
    y = cast(x, dtype=torch.float8_e4m3fn, seed=913, offset=2**32 - 17)
    expected = oracle.cast(x.contiguous().numpy(), oracle.E4M3, 1, 913, 2**32 - 17)
    assert y.shape == x.shape
    assert np.array_equal(y.contiguous().view(torch.uint8).numpy().reshape(-1),
                          expected.reshape(-1))


def test_cuda_cast_option_validation(fake_launcher):
    from sr_states.cuda import cast as cuda_cast
    from sr_states.cuda import rn_cast_bf16, sr_cast_bf16

    with pytest.raises(TypeError, match="float32"):
        rn_cast_bf16(torch.ones(4, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="contiguous"):
        rn_cast_bf16(torch.ones(8)[::2])
    with pytest.raises(ValueError, match="block_size"):
        rn_cast_bf16(torch.ones(4), block_size=3)
    with pytest.raises(ValueError, match="num_warps"):
        sr_cast_bf16(torch.ones(4), seed=7, num_warps=3)
    with pytest.raises(ValueError, match="store_mode"):
        sr_cast_bf16(torch.ones(4), seed=7, store_mode="invalid")
    with pytest.raises(ValueError, match="contiguous"):
        cuda_cast(torch.ones(8)[::2], dtype=torch.float16)
    out = sr_cast_bf16(torch.ones(5), seed=1)
    assert out.dtype == torch.bfloat16 and out.shape == (5,)


@pytest.mark.parametrize("kwargs", [{"lr": -1}, {"lr": float("nan")}, {"eps": -1},
                                    {"eps": float("inf")}, {"betas": (0.9, 1)},
                                    {"betas": (float("nan"), 0.9)}, {"weight_decay": -1},
                                    {"state_dtype": torch.int32}, {"rounding": "invalid"},
                                    {"block_size": 64}])
def test_adamw_rejects_invalid_options(kwargs):
    with pytest.raises(ValueError):
        AdamWTriton([torch.nn.Parameter(torch.ones(1))], **kwargs)


@pytest.mark.parametrize(("kwargs", "message"), [({"lr": -0.1}, "learning rate"),
                                                 ({"lr": 0.1, "momentum": 1.0}, "momentum value"),
                                                 ({"lr": 0.1, "rounding": "invalid"}, "rounding"),
                                                 ({"lr": 0.1, "block_size": 64}, "block_size")])
def test_sgdm_rejects_invalid_options(kwargs, message):
    with pytest.raises(ValueError, match=message):
        SGDMTriton([torch.nn.Parameter(torch.ones(4))], **kwargs)


@pytest.mark.parametrize("kind", ["sgdm", "adamw"])
def test_functional_validation(kind, fake_launcher):
    tensors = [torch.randn(257), torch.randn(257), torch.zeros(257, dtype=torch.bfloat16)]
    if kind == "adamw":
        tensors.append(torch.zeros(257, dtype=torch.bfloat16))
        function = cuda_adamw_step_
        options = dict(lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=1e-2, step=1,
                       seed=0)
    else:
        function = cuda_sgdm_step_
        options = dict(lr=1e-3, momentum_factor=0.9, seed=0)
    with pytest.raises(ValueError, match="overlap"):
        function(tensors[0], tensors[0], *tensors[2:], **options)
    with pytest.raises(ValueError, match="identical shapes"):
        function(tensors[0][:-1], *tensors[1:], **options)
    strided = [torch.zeros(514, dtype=t.dtype)[::2] for t in tensors]
    with pytest.raises(ValueError, match="contiguous"):
        function(*strided, **options)
    with pytest.raises(TypeError, match="FP32 or BF16"):
        function(tensors[0].double(), *tensors[1:], **options)
    if kind == "adamw":
        with pytest.raises(ValueError, match="positive integer"):
            function(*tensors, **{**options, "step": 0})
        with pytest.raises(ValueError, match="state dtype"):
            function(*tensors[:-1], tensors[-1].float(),
                     formats=(StateFormat(torch.bfloat16), StateFormat(torch.bfloat16)),
                     **options)
    assert not fake_launcher.calls
    function(*tensors, **options)
    assert len(fake_launcher.calls) == 1


def test_native_launcher_refuses_cpu_for_the_fused_step():
    p = torch.nn.Parameter(torch.ones(3))
    p.grad = torch.ones(3)
    opt = AdamWReferenceSR([p])
    with pytest.raises(ValueError, match="require CUDA tensors"):
        opt.step()
    assert opt._rng_step() == 1 and "exp_avg" in opt.state[p]


@pytest.mark.parametrize("cls", CLASSES)
@pytest.mark.parametrize("state_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("parameter_dtype", [torch.float32, torch.bfloat16])
def test_checkpoint_keeps_state_precision(cls, state_dtype, parameter_dtype):
    p = torch.nn.Parameter(torch.ones(4, dtype=parameter_dtype))
    opt = cls([p], lr=0.01, state_dtype=state_dtype, seed=42)
    original = torch.tensor([0.0, -0.0, 1.003125, 0.503125], dtype=state_dtype)
    for name in opt._state_names:
        opt.state[p][name] = original.clone()
    if "exp_avg" in opt._state_names:
        opt.state[p]["step"] = 7
    opt.param_groups[0]["sr_step"] = 2**32 + 31
    checkpoint = copy.deepcopy(opt.state_dict())
    q = torch.nn.Parameter(p.detach().clone())
    restored = cls([q], lr=0.3, state_dtype=torch.float32, seed=99)
    seen = []
    restored.register_load_state_dict_post_hook(
        lambda o: seen.append(o.state[q][o._state_names[0]].dtype))
    restored.load_state_dict(checkpoint)
    assert seen == [state_dtype]
    for name in opt._state_names:
        actual = restored.state[q][name]
        assert actual.dtype == state_dtype
        bits = torch.int32 if state_dtype == torch.float32 else torch.int16
        assert torch.equal(actual.view(bits), original.view(bits))
        assert actual.data_ptr() != checkpoint["state"][0][name].data_ptr()
    assert restored.param_groups[0]["sr_step"] == 2**32 + 31
    assert restored.param_groups[0]["sr_seed"] == 42
    if "exp_avg" in opt._state_names:
        assert restored.state[q]["step"] == 7


def test_legacy_checkpoint_drops_sr_offset_and_restarts_rng():
    p = torch.nn.Parameter(torch.ones(5))
    opt = AdamWReferenceSR([p], seed=5)
    checkpoint = copy.deepcopy(opt.state_dict())
    group = checkpoint["param_groups"][0]
    del group["sr_step"]
    group["sr_offset"] = 2**32 + 29
    resumed = AdamWReferenceSR([torch.nn.Parameter(torch.ones(5))], seed=7)
    resumed.load_state_dict(checkpoint)
    assert resumed.param_groups[0]["sr_step"] == 0
    assert resumed.param_groups[0]["sr_seed"] == 5
    assert "sr_offset" not in resumed.param_groups[0]
    assert group["sr_offset"] == 2**32 + 29  # the caller's checkpoint is untouched


def test_checkpoint_before_first_step_keeps_state_lazy():
    opt = SGDMTriton([torch.nn.Parameter(torch.ones(4))], lr=0.1)
    opt.load_state_dict(copy.deepcopy(opt.state_dict()))
    assert not opt.state


@pytest.mark.parametrize("rn,sr", [(AdamWReferenceRN, AdamWReferenceSR),
                                   (SGDMReferenceRN, SGDMReferenceSR)])
def test_rn_classes_force_nearest_in_overrides_and_checkpoints(rn, sr):
    dtypes = (torch.float8_e4m3fn, torch.float8_e5m2)
    per_state = {n: StateFormat(d) for n, d in zip(rn._state_names, dtypes)}
    nearest = {n: StateFormat(d, "nearest") for n, d in zip(rn._state_names, dtypes)}
    opt = rn([torch.nn.Parameter(torch.ones(3))], lr=0.01, state_format=per_state, seed=5)
    expected = sr([torch.nn.Parameter(torch.ones(3))], lr=0.01, state_format=nearest, seed=5)
    assert opt.param_groups[0]["state_format"] == expected.param_groups[0]["state_format"]
    for override in ({"state_format": StateFormat(torch.bfloat16)}, {"rounding": "stochastic"}):
        opt.add_param_group({"params": [torch.nn.Parameter(torch.ones(2))], **override})
        assert all(f["rounding"] == "nearest"
                   for f in opt.param_groups[-1]["state_format"].values())
    checkpoint = copy.deepcopy(expected.state_dict())
    for fmt in checkpoint["param_groups"][0]["state_format"].values():
        fmt["rounding"] = "stochastic"
    resumed = rn([torch.nn.Parameter(torch.ones(3))], lr=0.01)
    resumed.load_state_dict(checkpoint)
    assert resumed.param_groups[0]["state_format"] == expected.param_groups[0]["state_format"]


@pytest.mark.parametrize("cls", CLASSES)
def test_unregistered_rule_in_override_or_checkpoint_is_rejected(cls):
    p = torch.nn.Parameter(torch.ones(1))
    with pytest.raises(ValueError, match="rounding"):
        cls([{"params": [p], "rounding": "missing"}], lr=0.1)
    opt = cls([p], lr=0.1)
    checkpoint = copy.deepcopy(opt.state_dict())
    checkpoint["param_groups"][0]["state_format"][cls._state_names[0]]["rounding"] = "missing"
    with pytest.raises(ValueError, match="rounding"):
        opt.load_state_dict(checkpoint)
    assert opt.param_groups[0]["state_format"][cls._state_names[0]]["rounding"] == "stochastic"


class ThreeState(StateOptimizer):
    """A user optimizer supplying only FP32 math (per-parameter base path)."""

    _state_names = ("a", "b", "c")

    def __init__(self, params, **kwargs):
        super().__init__(params, {"lr": 0.01}, **kwargs)

    def _compute(self, p32, g32, states32, group, step):
        a, b, c = states32
        a = a * 0.8 + g32
        b = b * 0.5 + g32.square()
        c = c + g32 * 0.1
        return p32 - group["lr"] * (a + b + c), (a, b, c)


def test_user_optimizer_with_fp32_states_and_checkpoint():
    formats = {"a": StateFormat(torch.float32), "b": StateFormat(torch.float32, "nearest"),
               "c": StateFormat(torch.float32)}
    p = torch.nn.Parameter(torch.ones(13))
    opt = ThreeState([p], state_format=formats, seed=71)
    p.grad = torch.linspace(-1, 1, 13)
    opt.step()
    q = torch.nn.Parameter(p.detach().clone())
    resumed = ThreeState([q])
    resumed.load_state_dict(copy.deepcopy(opt.state_dict()))
    for step in range(3):
        p.grad = q.grad = torch.sin(torch.arange(13) + step)
        opt.step()
        resumed.step()
        assert torch.equal(p, q)
    assert opt._rng_step() == 4


def test_user_optimizer_uses_builtin_casts_through_the_kernel(fake_launcher):
    p = torch.nn.Parameter(torch.ones(13))
    opt = ThreeState([p], state_format=StateFormat(torch.float8_e4m3fn), seed=71)
    p.grad = torch.linspace(-1, 1, 13)
    opt.step()
    assert [c[0] for c in fake_launcher.calls] == ["cast"] * 3
    assert all(opt.state[p][n].dtype == torch.float8_e4m3fn for n in "abc")


def test_update_keys_and_words():
    assert update_key(0, 1, 0) == 0x7D2B5EA8
    assert update_key(0xFEDCBA9876543210 + (1 << 64), (1 << 64) + 5, 3) == update_key(
        0xFEDCBA9876543210, 5, 3)
    for value in (0, 1, 16, -1, 2**31, 2**63 + 7, 2**90 + 2**33 + 4):
        lo, hi = split_words(value)
        assert 0 <= lo < 2**32 and 0 <= hi < 2**32
        assert (hi << 32) | lo == value % 2**64


def test_dtensor_parameters_are_rejected():
    import torch.distributed as dist
    from torch.distributed.tensor import DeviceMesh, DTensor, Replicate

    pytest.importorskip("torch.testing._internal.distributed.fake_pg")
    dist.init_process_group("fake", store=dist.HashStore(), rank=0, world_size=1)
    try:
        mesh = DeviceMesh("cpu", [0])
        value = DTensor.from_local(torch.ones(3), mesh, [Replicate()])
        p = torch.nn.Parameter(value)
        p.grad = value.clone()
        opt = SGDMReferenceSR([p], lr=0.01)
        with pytest.raises(NotImplementedError, match="DTensor.*FSDP2"):
            opt.step()
        assert p not in opt.state
    finally:
        dist.destroy_process_group()
