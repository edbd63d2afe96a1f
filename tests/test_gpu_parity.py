"""GPU parity: the native operator against the float64 oracle and the golden
vectors produced by the reference, on the fixture shapes and the BASELINE
configurations (full size where the oracle is fast, sampled heads otherwise).
"""
import math

import pytest
import torch

from ca_testlib import (assert_fp32_parity, assert_lowp_parity, cosine, gen_inputs, load_cfg1,
                        load_small_cases, norm_max_err, oracle, run_op)

pytestmark = pytest.mark.gpu

LOWP = [torch.bfloat16, torch.float16]


@pytest.mark.parametrize("impl", ["simt", "auto"])
def test_golden_small_cases_fp32(impl):
    for name, inp, exp in load_small_cases():
        outs, _ = run_op(*inp, dtype=torch.float32, impl=impl)
        assert_fp32_parity(outs, exp, tag=f"{name}[{impl}]")


@pytest.mark.parametrize("dtype", LOWP)
@pytest.mark.parametrize("impl", ["simt", "auto"])
def test_golden_small_cases_lowp(dtype, impl):
    for name, inp, _ in load_small_cases():
        q, k, v, lg, dy = inp
        outs, used = run_op(q, k, v, lg, dy, dtype=dtype, impl=impl)
        ref = oracle(used[0], used[1], used[2], lg, used[3])
        assert_lowp_parity(outs, ref, tag=f"{name}[{impl},{dtype}]", lowp_dtype=dtype)


def test_config1_fp32_golden():
    # [2,4,256,32] fp32, seed 0, gain 1, vs reference float64 outputs
    inp, exp = load_cfg1()
    outs, _ = run_op(*inp, dtype=torch.float32)
    assert_fp32_parity(outs, exp, tag="config1")


def test_config5_fixed_tau_fp32():
    # [64,4,256,64] fp32, seed 1, fixed tau = 0.30
    q, k, v, dy = gen_inputs((64, 4, 256, 64), 1)
    lg = torch.full((4,), math.log(1 / 0.30))
    outs, _ = run_op(q, k, v, lg, dy, dtype=torch.float32)
    ref = oracle(q, k, v, lg, dy)
    assert_fp32_parity(outs, ref, tag="config5")


def _head_subset_ref(used, lg, heads):
    q, k, v, dy = used
    sub = [t[:, heads] for t in (q, k, v, dy)]
    return oracle(sub[0], sub[1], sub[2], lg[heads], sub[3])


@pytest.mark.parametrize("impl,dtype", [("auto", torch.bfloat16), ("simt", torch.bfloat16),
                                        ("auto", torch.float16)])
def test_config2_sampled_heads(impl, dtype):
    # [2,16,2048,64] bf16, q,k,v,dy ~ N(0,1), gain 1; oracle on 2 heads x 2 batches.
    # The fp16 case pins the tensor-core forward's single-fp16 P at full length.
    q, k, v, dy = gen_inputs((2, 16, 2048, 64), 2)
    lg = torch.zeros(16)
    outs, used = run_op(q, k, v, lg, dy, dtype=dtype, impl=impl)
    heads = [0, 11]
    y, rdq, rdk, rdv, rdg = _head_subset_ref(used, lg, heads)
    o, o32, dq, dk, dv, dg = outs
    sub = lambda t: t[:, heads]
    assert_lowp_parity((sub(o), sub(o32), sub(dq), sub(dk), sub(dv), dg[heads]),
                       (y, rdq, rdk, rdv, rdg), tag=f"config2[{impl},{dtype}]", lowp_dtype=dtype)


@pytest.mark.parametrize("dtype", LOWP)
@pytest.mark.parametrize("T", [1024, 4096])
def test_config3_stress_sampled_heads(T, dtype):
    # [1,16,T,64] bf16, score std ~4, 10% adjacent keys duplicated (delta = 0);
    # also in fp16 (single-fp16 P in the tensor-core forward)
    q, k, v, dy = gen_inputs((1, 16, T, 64), 3000 + T, qk_mag=2.0, dup_frac=0.1)
    lg = torch.zeros(16)
    outs, used = run_op(q, k, v, lg, dy, dtype=dtype)
    heads = [3]
    y, rdq, rdk, rdv, rdg = _head_subset_ref(used, lg, heads)
    o, o32, dq, dk, dv, dg = outs
    sub = lambda t: t[:, heads]
    assert_lowp_parity((sub(o), sub(o32), sub(dq), sub(dk), sub(dv), dg[heads]),
                       (y, rdq, rdk, rdv, rdg), tag=f"config3 T={T} {dtype}", lowp_dtype=dtype)


def test_fp32_and_lowp_paths_agree_on_larger_shape():
    q, k, v, dy = gen_inputs((1, 2, 777, 64), 77)
    lg = torch.tensor([0.0, math.log(1 / 0.3)])
    o32, _ = run_op(q, k, v, lg, dy, dtype=torch.float32)
    obf, _ = run_op(q, k, v, lg, dy, dtype=torch.bfloat16)
    for a, b in zip(o32[2:], obf[2:]):
        assert cosine(b, a) > 0.999


def test_simt_and_auto_agree_bf16():
    q, k, v, dy = gen_inputs((2, 3, 700, 64), 5)
    lg = torch.tensor([0.0, 0.4, -0.3])
    a, _ = run_op(q, k, v, lg, dy, dtype=torch.bfloat16, impl="simt")
    b, _ = run_op(q, k, v, lg, dy, dtype=torch.bfloat16, impl="auto")
    assert norm_max_err(b[1], a[1]) < 1e-4
    for x, y in zip(b[2:], a[2:]):
        assert cosine(x, y) > 0.9999


@pytest.mark.parametrize("shape", [(3, 37, 384, 64), (5, 60, 256, 64), (1, 1, 129, 64), (2, 80, 640, 64)])
def test_persistent_backward_schedules_agree_with_simt(shape):
    # Work-item counts from far below to far above the SM count (333, 600, 2 and 800 items
    # of one to five query tiles): every item of the persistent tcgen05 backward must
    # agree with the CUDA-core path, which schedules one block per tile.
    B, H, T, D = shape
    q, k, v, dy = gen_inputs(shape, 91 + T)
    g = torch.Generator().manual_seed(T)
    lg = torch.randn(H, generator=g) * 0.3
    a, _ = run_op(q, k, v, lg, dy, dtype=torch.bfloat16, impl="simt")
    b, _ = run_op(q, k, v, lg, dy, dtype=torch.bfloat16, impl="tcgen05")
    assert norm_max_err(b[1], a[1]) < 1e-4
    for name, x, y in zip(("dq", "dk", "dv", "dlog_gain"), b[2:], a[2:]):
        assert cosine(x, y) > 0.9999, name
