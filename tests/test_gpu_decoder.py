"""GPU tests of the CA-S decoder on the native operator: the reference's full
decoder causality check (cuda/benchmark.py:85-105: 101M model, T=2048, future
bytes changed, earlier logits bit-identical) and a finite, decreasing loss over a
few AdamW steps."""
import pytest
import torch

from continuum_attention_b200.decoder import ContinuumDecoderConfig, ContinuumDecoderLM, count_parameters
from continuum_attention_b200.distributed import build_adamw, train_step

pytestmark = pytest.mark.gpu


def test_full_decoder_causality_bitwise():
    torch.manual_seed(4242)
    model = ContinuumDecoderLM(ContinuumDecoderConfig(ca_query_tile=128)).cuda().eval()
    assert count_parameters(model)["total"] == 101205120
    ids = torch.randint(0, 256, (1, 2048), device="cuda")
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        base = model(ids)["logits"]
        for cut in (127, 1023, 1024, 2046):
            edited = ids.clone()
            edited[:, cut + 1:] = torch.randint_like(edited[:, cut + 1:], 0, 256)
            changed = model(edited)["logits"]
            assert torch.equal(base[:, :cut + 1], changed[:, :cut + 1]), f"decoder leak at cut {cut}"


def test_training_steps_reduce_loss():
    torch.manual_seed(0)
    cfg = ContinuumDecoderConfig(block_size=512, d_model=256, n_heads=4, n_layers=2)
    model = ContinuumDecoderLM(cfg).cuda()
    opt = build_adamw(model, lr=2e-3)
    g = torch.Generator(device="cpu").manual_seed(1)
    # a learnable stream: repeated random 64-byte pattern
    pat = torch.randint(0, 256, (64,), generator=g)
    batch = pat.repeat(4, 8).cuda()
    losses = [train_step(model, opt, batch).item() for _ in range(8)]
    assert all(torch.isfinite(torch.tensor(losses)))
    assert losses[-1] < losses[0] - 0.5
    gains = torch.stack([b.attn.log_qk_gain.detach() for b in model.blocks])
    assert gains.abs().sum() > 0          # the learned gains moved


def test_linear_weight_grad_in_fp32_matches_autocast_linear():
    from continuum_attention_b200.decoder import Linear
    torch.manual_seed(3)
    ours = Linear(256, 512, bias=False).cuda()
    ref = torch.nn.Linear(256, 512, bias=False).cuda()
    ref.weight.data.copy_(ours.weight.data)
    x = torch.randn(4, 96, 256, device="cuda")
    dy = torch.randn(4, 96, 512, device="cuda")
    outs = []
    for m in (ours, ref):
        xi = x.clone().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = m(xi)
        y.backward(dy.to(y.dtype))
        outs.append((y, xi.grad, m.weight.grad))
    (y1, dx1, dw1), (y2, dx2, dw2) = outs
    assert y1.dtype == y2.dtype == torch.bfloat16
    assert torch.equal(y1, y2)                       # the same bf16 product as autocast
    assert torch.equal(dx1, dx2)
    assert dw1.dtype == torch.float32
    # autocast's dW is the bf16 rounding of the fp32 accumulator this one keeps
    exact = (dy.to(torch.bfloat16).double().reshape(-1, 512).t() @ x.to(torch.bfloat16).double().reshape(-1, 256))
    assert ((dw1.double() - exact).abs() <= 1e-5 * exact.abs().max()).all()
    assert ((dw2.double() - dw1.double()).abs() <= 2 ** -8 * dw1.double().abs() + 1e-6).all()


def test_clip_folded_into_fused_adamw_matches_clip_grad_norm():
    from continuum_attention_b200.distributed import clip_and_step
    torch.manual_seed(5)
    cfg = ContinuumDecoderConfig(block_size=256, d_model=128, n_heads=2, n_layers=1)
    a = ContinuumDecoderLM(cfg).cuda()
    b = ContinuumDecoderLM(cfg).cuda()
    b.load_state_dict(a.state_dict())
    oa, ob = build_adamw(a, lr=1e-2), build_adamw(b, lr=1e-2)
    batch = torch.randint(0, 256, (2, 256), device="cuda")
    for step in range(3):
        oa.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = a(batch, targets=batch)["loss"]
        loss.backward()
        for pa, pb in zip(a.parameters(), b.parameters()):   # the same gradients on both sides
            pb.grad = None if pa.grad is None else pa.grad.clone()
        clip_and_step(a, oa, 0.05)                             # folded: the norm is far above 0.05
        torch.nn.utils.clip_grad_norm_(b.parameters(), 0.05)
        ob.step()
        for (n, pa), pb in zip(a.named_parameters(), b.parameters()):
            err = (pa - pb).abs().max().item()
            assert err <= 1e-6 * max(pb.abs().max().item(), 1.0), (step, n, err)
