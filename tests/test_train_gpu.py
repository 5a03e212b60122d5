"""A Qwen2-shaped training step with every nn.Linear on the protected NVFP4
path (forward, dgrad and wgrad GEMMs through the ABFT engine): one
accumulator fault in one GEMM is detected and recomputed, every other GEMM
is clean, and loss and gradients stay finite and match the unprotected NVFP4
step bit for bit."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _model(fault=None, protected=True):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    from sdc_b200.gemm.linear import install

    torch.manual_seed(0)
    cfg = Qwen2Config(num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=1024, max_position_embeddings=512, rope_theta=1e6,
                      tie_word_embeddings=True, attn_implementation="sdpa")
    model = Qwen2ForCausalLM(cfg).to(DEV)
    abft = {"method": "classic", "implementation": "native", "reference_mode": "input_fused",
            "reference_layout": "kslice", "on_error": "report", "recovery": "recompute", "locate": True,
            "atol": 1e-3, "rtol": 1e-4} if protected else None
    install(model, "nvfp4", "block16", abft_config=abft, fault_config=fault, report_max_records=256)
    return model


def _step(model):
    tokens = torch.randint(0, 1024, (2, 128), device=DEV, generator=torch.Generator(device=DEV).manual_seed(1))
    with torch.autocast("cuda", dtype=torch.bfloat16):
        loss = model(input_ids=tokens, labels=tokens).loss
    loss.backward()
    grads = {name: p.grad.detach().clone() for name, p in model.named_parameters() if p.grad is not None}
    return loss.detach(), grads


def test_protected_training_step_detects_locates_and_recovers_one_fault():
    from sdc_b200.gemm.linear import ProtectedLinear

    fault = {"location": "accumulator", "row": 5, "col": 7, "bit": 26, "call_index": 1}
    model = _model(fault)
    loss, grads = _step(model)
    protection = next(m.protection for m in model.modules() if isinstance(m, ProtectedLinear))
    reports = list(protection.reports)
    # 2 layers x 7 linears + the tied LM head, 3 GEMMs each.
    assert len(reports) == protection.call_index == (2 * 7 + 1) * 3
    roles = {report.context["role"] for report in reports}
    assert roles == {"forward", "dgrad", "wgrad"}
    detected = [r for r in reports if bool(r.detected)]
    assert len(detected) == 1, [r.context for r in detected]
    first = detected[0]
    assert first.context["call_index"] == 1 and first.context["role"] == "forward"
    assert first.context["layer"] == "model.layers.0.self_attn.q_proj"
    # The Classic locator only names the element when the flip dominates the
    # row-weighted channel's threshold; a located error is the injected one.
    if bool(first.located):
        assert first.location.tolist() == [5, 7]
    assert bool(first.recovered) and first.context["recovery_action"] == "full_recompute"
    assert torch.isfinite(loss)
    assert all(torch.isfinite(g).all() for g in grads.values())

    # The recomputed step equals an unprotected NVFP4 step bit for bit.
    plain_loss, plain_grads = _step(_model(protected=False))
    assert torch.equal(loss, plain_loss)
    assert grads.keys() == plain_grads.keys()
    assert all(torch.equal(grads[k], plain_grads[k]) for k in grads)
