"""TinyLM (architecture.py:204-245) with the B200 operator in its continuous
variants: logits and gradients against the same model whose attention is the
float64 oracle restatement, and the CUDA-graph training step against eager steps."""
import copy

import pytest
import torch

from cpu_attention import cpu_continuum_attention
from continuum_attention_b200.tinylm import TinyLM, TinyLMTrainer, build_optimizer, train_step

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("variant", ["P", "S", "H", "R"])
def test_tinylm_matches_float64_oracle_attention(variant):
    torch.manual_seed(7)
    model = TinyLM(variant=variant, seq_len=96, width=128, hidden=160, heads=4).cuda()
    if variant in ("S", "H"):
        with torch.no_grad():
            for i in range(6):
                getattr(model, f"b{i}").attn.log_qk_gain.add_(torch.linspace(-0.3, 0.4, 4, device="cuda"))
    ref = copy.deepcopy(model).double()
    for i in range(6):
        getattr(ref, f"b{i}").attn.attention_fn = cpu_continuum_attention
    x = torch.randint(0, 256, (3, 96), device="cuda")
    logits = model(x)
    logits_ref = ref(x)
    err = (logits.double() - logits_ref).abs().max() / logits_ref.abs().max()
    assert err < 1e-5, err.item()
    loss = torch.nn.functional.cross_entropy(logits.reshape(-1, 256), x.reshape(-1))
    loss_ref = torch.nn.functional.cross_entropy(logits_ref.reshape(-1, 256), x.reshape(-1))
    loss.backward()
    loss_ref.backward()
    for (name, p), p_ref in zip(model.named_parameters(), ref.parameters()):
        g, gr = p.grad.double(), p_ref.grad
        rel = (g - gr).abs().max() / gr.abs().max().clamp_min(1e-30)
        assert rel < 1e-4, (name, rel.item())


def test_graph_captured_training_matches_eager():
    torch.manual_seed(3)
    base = TinyLM(variant="S", seq_len=64, width=64, hidden=96, heads=4).cuda()
    eager = copy.deepcopy(base)
    opt = build_optimizer(eager)
    trainer = TinyLMTrainer(copy.deepcopy(base), batch_size=4, seq_len=64)
    g = torch.Generator(device="cpu").manual_seed(11)
    batches = [torch.randint(0, 256, (4, 65), generator=g).cuda() for _ in range(4)]
    for b in batches:
        le = float(train_step(eager, opt, b[:, :-1], b[:, 1:]))
        lg = float(trainer.step(b[:, :-1], b[:, 1:]))
        assert abs(le - lg) <= 1e-5 * abs(le), (le, lg)
    for p, q in zip(eager.parameters(), trainer.model.parameters()):
        assert torch.allclose(p, q, rtol=1e-4, atol=1e-6)


def test_reference_size_tinylm_trains_with_graph():
    torch.manual_seed(1729)
    model = TinyLM(variant="P").cuda()
    trainer = TinyLMTrainer(model, batch_size=8, seq_len=192)
    x = torch.randint(0, 256, (8, 193), device="cuda")
    losses = [float(trainer.step(x[:, :-1], x[:, 1:])) for _ in range(20)]
    assert losses[-1] < losses[0] - 0.5, losses
