"""Work order over head-sequences in the tensor-core kernels.

At T >= 4096 both kernels hand out their work in groups of 16 head-sequences
(heaviest first inside each group), so that the CTAs running together share the
tiles they read in L2.  The order changes nothing that a head-sequence computes:
with the deterministic backward every output is bitwise the same whether a
head-sequence runs inside a group, in another grouping, or alone.
"""
import os
import subprocess
import sys

import pytest
import torch

import continuum_attention_b200 as ca
from ca_testlib import gen_inputs

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _run(q, k, v, lg, dy):
    q, k, v, lg = (t.detach().clone().requires_grad_(True) for t in (q, k, v, lg))
    with ca.deterministic_backward():
        y = ca.continuum_attention(q, k, v, lg, 128)
        grads = torch.autograd.grad((y.float() * dy.float()).sum(), (q, k, v, lg))
    return [y.detach()] + list(grads)


def _inputs(shape, seed):
    q, k, v, dy = (t.to("cuda", torch.bfloat16) for t in gen_inputs(shape, seed, qk_mag=2.0, dup_frac=0.1))
    lg = torch.linspace(-0.3, 0.2, shape[1], device="cuda")
    return q, k, v, lg, dy


def test_grouped_order_matches_slices_bitwise():
    # [1,40,4096,64]: 32 query tiles, so groups of 16, 16 and 8 head-sequences
    q, k, v, lg, dy = _inputs((1, 40, 4096, 64), 61)
    full = _run(q, k, v, lg, dy)
    for a, b in ((0, 8), (13, 21), (32, 40)):   # ungrouped slices (8 head-sequences: one group)
        part = _run(q[:, a:b], k[:, a:b], v[:, a:b], lg[a:b], dy[:, a:b])
        for name, x, y in zip(("y", "dq", "dk", "dv"), full[:4], part[:4]):
            assert torch.equal(x[:, a:b], y), (name, a, b)
        assert torch.equal(full[4][a:b], part[4]), ("dlog_gain", a, b)


def test_group_size_override_matches_default_bitwise(tmp_path):
    # a ragged grouping (3, 3, 3, 1 head-sequences) in a child process, against the
    # default single group here
    out = tmp_path / "grouped.pt"
    code = (
        "import sys, torch; sys.path.insert(0, %r); sys.path.insert(0, %r)\n"
        "import test_gpu_head_groups as t\n"
        "torch.save([x.cpu() for x in t._run(*t._inputs((2, 5, 1024, 64), 62))], %r)\n"
    ) % (HERE, os.path.dirname(HERE), str(out))
    env = dict(os.environ, CA_B200_HEAD_GROUP="3")
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    grouped = torch.load(out)
    here = _run(*_inputs((2, 5, 1024, 64), 62))
    for name, x, y in zip(("y", "dq", "dk", "dv", "dlog_gain"), here, grouped):
        assert torch.equal(x.cpu(), y), name
