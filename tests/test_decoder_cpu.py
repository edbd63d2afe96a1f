"""CPU tests of the CA-S decoder wiring (cuda/test_cpu.py:25-27 pattern, the
decoder causality check of cuda/continuum_attention.py:1490-1502)."""
import pytest
import torch

from continuum_attention_b200.decoder import ContinuumDecoderConfig, ContinuumDecoderLM, count_parameters
from cpu_attention import cpu_continuum_attention


def test_parameter_budget_matches_reference():
    model = ContinuumDecoderLM(ContinuumDecoderConfig())
    assert count_parameters(model) == {"total": 101205120, "trainable": 101205120}
    gains = sum(b.attn.log_qk_gain.numel() for b in model.blocks)
    assert gains == 8 * 16
    assert model.lm_head.weight.data_ptr() != model.byte_emb.weight.data_ptr()   # untied


def test_config_validation():
    with pytest.raises(ValueError):
        ContinuumDecoderConfig(d_model=100, n_heads=16)
    with pytest.raises(ValueError):
        ContinuumDecoderConfig(d_model=48, n_heads=16)      # odd head dim
    with pytest.raises(ValueError):
        ContinuumDecoderConfig(dropout=0.1)


def _tiny(seed=0):
    torch.manual_seed(seed)
    cfg = ContinuumDecoderConfig(block_size=32, d_model=64, n_heads=4, n_layers=2)
    return ContinuumDecoderLM(cfg, attention_fn=cpu_continuum_attention)


def test_forward_loss_and_gain_gradients():
    model = _tiny()
    ids = torch.randint(0, 256, (2, 24))
    out = model(ids, targets=ids)
    assert out["logits"].shape == (2, 24, 256)
    out["loss"].backward()
    for b in model.blocks:
        assert b.attn.log_qk_gain.grad is not None
        assert torch.isfinite(b.attn.log_qk_gain.grad).all()
        assert b.attn.log_qk_gain.grad.abs().sum() > 0


def test_decoder_is_causal():
    model = _tiny().eval()
    T = 32
    x = torch.randint(0, 256, (1, T))
    x2 = x.clone()
    x2[:, T // 2 + 1:] = torch.randint(0, 256, (1, T - T // 2 - 1))
    with torch.no_grad():
        a, b = model(x)["logits"], model(x2)["logits"]
    assert (a[:, :T // 2 + 1] - b[:, :T // 2 + 1]).abs().max().item() <= 1e-5


def test_linear_is_nn_linear_off_the_bf16_cuda_path():
    # decoder.Linear keeps nn.Linear's parameters and state-dict keys; outside bf16
    # autocast on CUDA it is nn.Linear itself
    from continuum_attention_b200.decoder import Linear
    torch.manual_seed(2)
    ours, ref = Linear(16, 8, bias=False), torch.nn.Linear(16, 8, bias=False)
    ref.load_state_dict(ours.state_dict())
    assert list(ours.state_dict()) == list(ref.state_dict())
    x = torch.randn(3, 16, requires_grad=True)
    xr = x.detach().clone().requires_grad_(True)
    ours(x).sum().backward()
    ref(xr).sum().backward()
    assert torch.equal(x.grad, xr.grad) and torch.equal(ours.weight.grad, ref.weight.grad)


def test_clip_and_step_matches_clip_grad_norm_without_fused_adamw():
    from continuum_attention_b200.distributed import build_adamw, clip_and_step
    a, b = _tiny(1), _tiny(1)
    oa, ob = build_adamw(a, lr=1e-2), build_adamw(b, lr=1e-2)
    batch = torch.randint(0, 256, (2, 32))
    for m in (a, b):
        m(batch, targets=batch)["loss"].backward()
    clip_and_step(a, oa, 0.05)                 # CPU parameters: the unfused optimizer path
    torch.nn.utils.clip_grad_norm_(b.parameters(), 0.05)
    ob.step()
    for pa, pb in zip(a.parameters(), b.parameters()):
        assert torch.equal(pa, pb)


def test_matches_reference_decoder_on_cpu():
    """The reference ContinuumDecoderLM's own logits, loss and gradients (fixture made
    by tests/golden/make_golden.py), reproduced by this decoder on the CPU with the
    float64 oracle attention in place of the operator: pins the embedding, rotary
    convention, norms, residual wiring, untied head and loss."""
    from decoder_fixture import check, compare, load
    cfg, state, ids, logits, loss, grads = load()
    model = ContinuumDecoderLM(cfg, attention_fn=cpu_continuum_attention)
    model.load_state_dict(state)
    check(compare(model, ids, logits, loss, grads))
