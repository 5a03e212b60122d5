"""CPU contract tests of the Linear bridge and MethodSession mirrors.

As in the reference's own CPU tests (tests/cutlass_gemm/test_linear.py,
tests/abft/test_session.py), the GEMM entry is replaced by torch.mm so the
autograd plumbing, install semantics, role/call-index contexts and session
checkpoints are checked without a GPU.
"""
import copy
import json
from types import SimpleNamespace

import pytest
import torch
from torch import nn
from torch.utils.checkpoint import checkpoint

import sdc_b200.abft as abft
from sdc_b200.abft import methods
from sdc_b200.abft.methods import AbftMethod
from sdc_b200.abft.session import MethodSession
from sdc_b200.gemm import backend
from sdc_b200.gemm.linear import CutlassLinear, ProtectedLinear, install, protection_sessions


@pytest.fixture
def bridge(monkeypatch):
    calls = []

    def mm(a, b):
        assert a.is_contiguous() or a.T.is_contiguous()
        assert b.is_contiguous() or b.T.is_contiguous()
        calls.append((a.dtype, b.dtype))
        return torch.mm(a, b)

    monkeypatch.setattr(backend, "mm", mm)
    return calls


# --- Linear bridge -------------------------------------------------------------------

@pytest.mark.parametrize("bias", [False, True])
@pytest.mark.parametrize("summed", [False, True])
def test_forward_backward_match_nn_linear(bridge, bias, summed):
    torch.manual_seed(11)
    original = nn.Linear(8, 16, bias=bias)
    reference = copy.deepcopy(original)
    layer = ProtectedLinear(original)
    x = torch.randn(2, 8, 3).transpose(1, 2).requires_grad_()
    xr = x.detach().clone().requires_grad_()
    actual, expected = layer(x), reference(xr)
    torch.testing.assert_close(actual, expected)
    grad = torch.randn_like(actual)
    (actual.sum() if summed else actual).backward(None if summed else grad)
    (expected.sum() if summed else expected).backward(None if summed else grad)
    torch.testing.assert_close(x.grad, xr.grad)
    torch.testing.assert_close(layer.weight.grad, reference.weight.grad)
    if bias:
        torch.testing.assert_close(layer.bias.grad, reference.bias.grad)
    assert len(bridge) == 3


def test_bf16_autocast_keeps_fp32_master_gradients(bridge):
    layer = ProtectedLinear(nn.Linear(8, 16))
    x = torch.randn(8, 8, requires_grad=True)
    with torch.autocast("cpu", dtype=torch.bfloat16):
        out = layer(x)
    out.sum().backward()
    assert out.dtype == torch.bfloat16
    assert bridge == [(torch.bfloat16, torch.bfloat16)] * 3
    assert layer.weight.dtype == layer.weight.grad.dtype == torch.float32
    assert layer.bias.grad.dtype == x.grad.dtype == torch.float32


def test_install_preserves_parameters_sharing_and_mode(bridge):
    shared = nn.Linear(8, 8).eval()
    tied = nn.Linear(8, 8)
    tied.weight = shared.weight
    model = nn.ModuleDict({"first": shared, "alias": shared, "tied": tied})
    parameters = list(model.parameters())
    install(model)
    assert model["first"] is model["alias"] and not model["first"].training
    assert model["first"].weight is model["tied"].weight
    assert all(a is b for a, b in zip(parameters, model.parameters(), strict=True))
    assert isinstance(install(nn.Linear(8, 8)), CutlassLinear)
    with pytest.raises(ValueError, match="no nn.Linear"):
        install(nn.ReLU())


@pytest.mark.parametrize("reentrant", [False, True])
def test_checkpoint_recomputation_gradients(bridge, reentrant):
    torch.manual_seed(12)
    layer = ProtectedLinear(nn.Linear(8, 8))
    reference = copy.deepcopy(layer)
    x = torch.randn(8, 8, requires_grad=True)
    xr = x.detach().clone().requires_grad_()
    checkpoint(layer, x, use_reentrant=reentrant).square().sum().backward()
    reference(xr).square().sum().backward()
    torch.testing.assert_close(x.grad, xr.grad)
    torch.testing.assert_close(layer.weight.grad, reference.weight.grad)
    assert len(bridge) >= 7


def test_small_transformer_all_linears_train(bridge):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    torch.manual_seed(13)
    config = Qwen2Config(vocab_size=32, hidden_size=16, intermediate_size=32, num_hidden_layers=1,
                         num_attention_heads=2, num_key_value_heads=2, max_position_embeddings=32)
    config._attn_implementation = "eager"
    model = Qwen2ForCausalLM(config)
    names = {name for name, module in model.named_modules() if isinstance(module, nn.Linear)}
    before = {name: model.get_submodule(name).weight.detach().clone() for name in names}
    install(model)
    assert "lm_head" in names and all(isinstance(model.get_submodule(n), ProtectedLinear) for n in names)
    optimizer = torch.optim.SGD(model.parameters(), lr=0.1)
    tokens = torch.randint(0, 32, (2, 8))
    loss = model(input_ids=tokens, labels=tokens).loss
    assert torch.isfinite(loss)
    loss.backward()
    optimizer.step()
    for name in names:
        layer = model.get_submodule(name)
        assert torch.isfinite(layer.weight.grad).all() and not torch.equal(layer.weight, before[name])


def test_backend_mm_rejects_cpu_before_any_kernel():
    with pytest.raises(RuntimeError, match="CUDA"):
        backend.mm(torch.ones(8, 8), torch.ones(8, 8))


@pytest.mark.parametrize("reentrant", [False, True])
def test_protected_roles_contexts_and_bounded_reports(monkeypatch, reentrant):
    calls = []

    class Report:
        def to_record(self):
            pytest.fail("in-memory reports must not synchronise")

    def execute(a, b, precision, scaling, global_scale, abft_config, fault_config, context, *, method_instance=None):
        calls.append(dict(context))
        assert abft_config.method == "classic" and method_instance is not None
        return a @ b, Report()

    monkeypatch.setattr(abft, "execute", execute)
    model = install(nn.Sequential(nn.Linear(8, 8)), abft_config={"method": "classic"}, report_max_records=2)
    x = torch.randn(8, 8, requires_grad=True)
    checkpoint(model, x, use_reentrant=reentrant).square().sum().backward()
    assert {c["role"] for c in calls} == {"forward", "dgrad", "wgrad"}
    assert [c["call_index"] for c in calls] == list(range(1, len(calls) + 1))
    assert all(c["layer"] == "0" and c["retry"] == 0 for c in calls)
    assert len(model[0].protection.reports) == 2
    assert protection_sessions(model)[0]["layers"] == ["0"]


def test_fault_only_protection_records_exception_reports(monkeypatch, tmp_path):
    class Report:
        def to_record(self):
            return {"detected": True}

    class Detection(RuntimeError):
        report = Report()

    def execute(a, b, precision, scaling, global_scale, abft_config, fault_config, context, *, method_instance=None):
        assert abft_config.method == "none" and method_instance is None
        assert fault_config.location == "accumulator"
        raise Detection("fault")

    monkeypatch.setattr(abft, "execute", execute)
    log = tmp_path / "reports.jsonl"
    model = install(nn.Linear(8, 8), fault_config={"location": "accumulator"}, report_max_records=1,
                    report_path=log)
    with pytest.raises(Detection) as caught:
        model(torch.ones(8, 8))
    assert model.protection.reports[0] is caught.value.report
    assert json.loads(log.read_text()) == {"detected": True}


# --- MethodSession ---------------------------------------------------------------------

class History(AbftMethod):
    stateful = True
    state_schema_version = 1

    def __init__(self):
        self.generator = torch.Generator().manual_seed(31)
        self.count = 0
        self.history = torch.zeros(8)

    def advance(self):
        sample = torch.rand((), generator=self.generator)
        self.history[self.count % 8] = sample
        self.count += 1
        return sample

    def prepare(self, operands, config, mm=None):
        raise NotImplementedError

    def propagate(self, partials, state):
        raise NotImplementedError

    def verify(self, observed, output, state, config):
        raise NotImplementedError

    def state_dict(self):
        return {"count": self.count, "history": self.history, "rng": self.generator.get_state()}

    def load_state_dict(self, state):
        self.count, self.history = state["count"], state["history"]
        self.generator.set_state(state["rng"])


@pytest.fixture
def history(monkeypatch):
    monkeypatch.setattr(methods, "_METHODS", dict(methods._METHODS))
    methods.register_method("history", History)
    return "history"


def call(session, *, shape=(3, 2, 4), precision="fp32", scaling="none", global_scale="amax",
         layer="model.layers.0.mlp", role="forward", dtype=torch.float32, device="cpu"):
    m, n, k = shape
    a = SimpleNamespace(ndim=2, shape=(m, k), device=torch.device(device), dtype=dtype)
    b = SimpleNamespace(ndim=2, shape=(k, n), device=torch.device(device), dtype=dtype)
    return session.call(a, b, precision, scaling, global_scale, layer, role)


def populate(session, **kwargs):
    with call(session, **kwargs) as (method, context):
        method.advance()
    return method, context


def test_same_profile_keeps_instance_and_counts_calls(history):
    session = MethodSession(history)
    with call(session) as (first, context):
        assert (context["call_index"], context["execution_kind"], context["retry"]) == (1, "forward_or_recompute", 0)
    with call(session) as (second, context):
        assert second is first and context["call_index"] == 2 and second.count == 0


@pytest.mark.parametrize("change", [{"layer": "other"}, {"role": "dgrad"}, {"role": "wgrad"}, {"shape": (5, 2, 4)},
                                    {"precision": "fp8", "scaling": "tensorwise"},
                                    {"precision": "nvfp4", "scaling": "block16"}, {"global_scale": 2.0},
                                    {"dtype": torch.bfloat16}])
def test_history_isolated_per_execution_profile(history, change):
    session = MethodSession(history)
    first, _ = populate(session)
    with call(session, **change) as (other, context):
        assert other is not first and other.count == 0
        assert context["execution_kind"] == ("backward" if change.get("role") else "forward_or_recompute")
    with call(session) as (again, _):
        assert again is first and again.count == 1


def test_checkpoint_round_trip_restores_history_rng_and_counter(history, tmp_path):
    session = MethodSession(history)
    populate(session)
    populate(session, role="dgrad")
    path = tmp_path / "session.pt"
    torch.save(session.state_dict(), path)
    expected = [populate(session)[0].advance().item() for _ in range(1)]
    restored = MethodSession(history)
    restored.load_state_dict(torch.load(path, weights_only=True))
    assert restored.call_index == 2
    assert [populate(restored)[0].advance().item() for _ in range(1)] == expected


def test_snapshot_does_not_alias_live_tensors(history):
    session = MethodSession(history)
    method, _ = populate(session)
    snapshot = session.state_dict()
    method.history.fill_(7)
    assert not torch.equal(snapshot["instances"][0]["state"]["history"], method.history)


def test_stateless_sessions_share_one_instance_without_scopes():
    session = MethodSession("classic")
    with call(session) as (first, _):
        pass
    with call(session, layer="x", role="wgrad", shape=(9, 9, 9)) as (second, context):
        assert second is first and context["call_index"] == 2
    payload = session.state_dict()
    assert payload["instances"] == [] and payload["pending_state"] is None
    fresh = MethodSession("classic")
    fresh.load_state_dict(payload)
    assert fresh.call_index == 2


def test_stateful_session_rejects_reentry(history):
    session = MethodSession(history)
    with call(session):
        with pytest.raises(RuntimeError, match="concurrent"):
            with call(session):
                pass
        with pytest.raises(RuntimeError, match="concurrent"):
            session.state_dict()


@pytest.mark.parametrize("field,value", [("schema_version", 2), ("call_index", -1), ("instances", {}),
                                         ("config_signature", "0" * 64)])
def test_malformed_checkpoint_rejected_and_live_state_kept(history, field, value):
    session = MethodSession(history)
    populate(session)
    payload = {**session.state_dict(), field: value}
    with pytest.raises(ValueError):
        session.load_state_dict(payload)
    assert session.call_index == 1


def test_config_change_rejected_on_restore(history):
    payload = MethodSession(history).state_dict()
    with pytest.raises(ValueError, match="does not match"):
        MethodSession({"method": history, "atol": 1.0}).load_state_dict(payload)


def test_generator_objects_cannot_enter_a_checkpoint(history, monkeypatch):
    session = MethodSession(history)
    method, _ = populate(session)
    monkeypatch.setattr(method, "state_dict", lambda: {"rng": method.generator})
    with pytest.raises(ValueError, match="generator"):
        session.state_dict()
