"""The CA-S decoder on the GPU against the reference model's own outputs.

The fixture (tests/golden/decoder_small.npz) holds the reference
ContinuumDecoderLM (cuda/continuum_attention.py:784-922) run on the CPU in
float32: its state dict, a batch of bytes, logits, loss and every parameter
gradient.  Here the same weights go into this repository's decoder on CUDA in
float32 (no autocast), so the native operator (fp32 CUDA-core kernels), the
fused rotary/QKV unpacking, the RMSNorm and GELU kernels all run, and the
results must match the reference to float32 rounding (tolerances in
tests/decoder_fixture.py)."""
import pytest
import torch

from continuum_attention_b200.decoder import ContinuumDecoderLM
from decoder_fixture import check, compare, load

pytestmark = pytest.mark.gpu


def test_decoder_matches_reference_model_fp32():
    cfg, state, ids, logits, loss, grads = load()
    model = ContinuumDecoderLM(cfg).cuda()
    model.load_state_dict(state)
    errs = compare(model, ids.cuda(), logits, loss, grads)
    print("DECODER_PARITY", {k: f"{v:.2e}" for k, v in errs.items()}, flush=True)
    check(errs)
