"""TinyLM with the CA operator: architecture, parameter budget and wiring on CPU
(the attention is the oracle-based stand-in; the GPU tests use the CUDA op)."""
import torch

from cpu_attention import cpu_continuum_attention
from continuum_attention_b200.tinylm import TinyLM, build_optimizer, parameters, train_step


def test_parameter_budget_and_state_dict_keys_match_reference():
    # architecture.py:204-245 and test_fusion.py:18-19
    for variant, count in [("B", 5008640), ("P", 5008640), ("R", 5008640), ("S", 5008664), ("H", 5008664)]:
        assert parameters(TinyLM(variant=variant)) == count
    keys = set(TinyLM(variant="S").state_dict())
    for k in ("tok_embed.weight", "pos_embed.weight", "b0.norm_attn.weight", "b0.attn.qkv.weight",
              "b0.attn.out.weight", "b0.attn.log_qk_gain", "b5.mlp.gate_up.weight", "b5.mlp.down.weight",
              "final_norm.weight", "lm_head.weight"):
        assert k in keys, k


def test_gain_parameters_and_training_step_on_cpu():
    torch.manual_seed(0)
    for variant in ("P", "S", "H", "R", "B", "F"):
        m = TinyLM(variant=variant, seq_len=24, width=32, hidden=48, heads=4,
                   attention_fn=cpu_continuum_attention)
        x = torch.randint(0, 256, (2, 24))
        opt = build_optimizer(m, lr=1e-2)
        losses = [float(train_step(m, opt, x, x)) for _ in range(4)]
        assert all(torch.isfinite(torch.tensor(losses)))
        assert losses[-1] < losses[0], (variant, losses)
        if variant in ("S", "H"):
            g = m.b0.attn.log_qk_gain
            assert g.grad is not None and torch.any(g.grad != 0)
