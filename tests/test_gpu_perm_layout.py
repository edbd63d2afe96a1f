"""The tensor-core forward's permuted key order (T a multiple of 16).

For T a multiple of 16 the tcgen05 forward reads K through a 5-D TMA view that puts
keys j and j+8 of each 16-key chunk side by side.  These cases cover the chunk, tile
and halo edges of that layout against the float64 oracle (forward and the backward
that follows it), and the permuted forward against the natural-order one
(``CA_B200_NO_PERM=1`` in a child process) on the same inputs.
"""
import os
import subprocess
import sys

import pytest
import torch

from ca_testlib import assert_lowp_parity, cosine, gen_inputs, norm_max_err, oracle, run_op

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("T", [16, 48, 144, 400, 1040])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_permuted_kernels_match_oracle(T, dtype):
    # one partial tile, chunk-aligned partial tiles, and T a multiple of 16 but not of 128
    q, k, v, dy = gen_inputs((1, 3, T, 64), 300 + T, qk_mag=1.5, dup_frac=0.1)
    lg = torch.tensor([0.0, 0.4, -0.4])
    outs, used = run_op(q, k, v, lg, dy, dtype=dtype, impl="tcgen05")
    ref = oracle(*used[:3], lg, used[3])
    assert_lowp_parity(outs, ref, tag=f"T={T} {dtype}", lowp_dtype=dtype)


def _child_outputs(path, shape, seed, env_extra):
    code = (
        "import sys, torch; sys.path.insert(0, %r); sys.path.insert(0, %r)\n"
        "from ca_testlib import gen_inputs, run_op\n"
        "q, k, v, dy = gen_inputs(%r, %d, qk_mag=2.0, dup_frac=0.1)\n"
        "lg = torch.linspace(-0.3, 0.3, %d)\n"
        "outs, _ = run_op(q, k, v, lg, dy, dtype=torch.bfloat16, impl='tcgen05')\n"
        "torch.save(outs, %r)\n"
    ) % (HERE, os.path.dirname(HERE), tuple(shape), seed, shape[1], str(path))
    env = dict(os.environ, **env_extra)
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    return torch.load(path)


def test_permuted_and_natural_orders_agree(tmp_path):
    # [2,4,2048,64] with the config-3 recipe: the two key orders compute the same
    # moments; only the order of the forward's sums over keys differs
    shape = (2, 4, 2048, 64)
    nat = _child_outputs(tmp_path / "nat.pt", shape, 77, {"CA_B200_NO_PERM": "1"})
    per = _child_outputs(tmp_path / "per.pt", shape, 77, {"CA_B200_NO_PERM": "0"})
    assert norm_max_err(per[1], nat[1]) < 1e-5
    for name, a, b in zip(("dq", "dk", "dv", "dlog_gain"), per[2:], nat[2:]):
        assert cosine(a, b) > 0.99999, name
    assert norm_max_err(per[5], nat[5]) < 1e-3


@pytest.mark.parametrize("T", [1, 2, 7, 15, 17, 31, 127, 129])
def test_tensor_core_kernels_at_tiny_and_odd_lengths(T):
    # the natural-order kernels (T not a multiple of 16) and one-tile edge cases of the
    # tensor-core path, against the float64 oracle
    q, k, v, dy = gen_inputs((2, 3, T, 64), 500 + T, qk_mag=1.5)
    lg = torch.tensor([0.0, 0.4, -0.4])
    outs, used = run_op(q, k, v, lg, dy, dtype=torch.bfloat16, impl="tcgen05")
    ref = oracle(*used[:3], lg, used[3])
    assert_lowp_parity(outs, ref, tag=f"T={T}")
