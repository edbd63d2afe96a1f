"""The reference's own CUDA extension, built from its sources, as a GPU comparison.

TEST INFRASTRUCTURE, like the rest of ``oracle/``: only tests import this module.
The product never loads what it builds.

The reference compiles its kernels at run time with ``load_inline`` from two
source strings embedded in ``cuda/continuum_attention.py`` (``_CUDA_CPP`` at
:35-63, ``_CUDA_SRC`` at :65-606; loader :608-620).  ``build_extension`` reads
those two strings out of the reference file (parsed with ``ast``, nothing of the
reference is executed), compiles them with the same ``load_inline`` call in a
temporary directory and keeps only the resulting extension module, as
``oracle/_ref/ca_ref_cuda.so`` (git-ignored; built where the reference project
is present, then shipped with the working tree).  The reference sources are not
copied into this repository.

``RefTiledCA`` restates the reference's tiled autograd op ``_CAExactTiled``
(cuda/continuum_attention.py:650-766) around the compiled kernels for two of
its modes:

* ``prefix_v6`` (fp16 inputs, T <= 2048; the mode of the reference's published
  V100 timing, README.md:97): per query tile the fp16 score GEMM, then
  ``scale_scores_half`` / ``forward_half`` and a W V GEMM (:670-690); backward
  ``backward_half_gw16`` and four GEMMs per tile accumulated in fp32 (:713-760);
* ``prefix`` (any dtype): fp32 scaled scores, ``forward`` (weights), and
  ``backward_fused`` (:734-736, 757-764).

Same call sequence, same dtypes, same per-tile accumulation, so timings and
outputs are the reference's.
"""
from __future__ import annotations

import ast
import glob
import importlib.machinery
import importlib.util
import os
import shutil
import tempfile

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
MODULE_NAME = "ca_ref_cuda"
SO_PATH = os.path.join(REF_DIR, MODULE_NAME + ".so")


def _source_strings(reference_root: str):
    path = os.path.join(reference_root, "cuda", "continuum_attention.py")
    tree = ast.parse(open(path).read(), filename=path)
    found = {}
    for node in tree.body:
        if isinstance(node, ast.Assign) and len(node.targets) == 1 and isinstance(node.targets[0], ast.Name):
            name = node.targets[0].id
            if name in ("_CUDA_CPP", "_CUDA_SRC") and isinstance(node.value, ast.Constant):
                found[name] = node.value.value
    if set(found) != {"_CUDA_CPP", "_CUDA_SRC"}:
        raise RuntimeError(f"{path}: extension source strings not found")
    return found["_CUDA_CPP"], found["_CUDA_SRC"], path


def build_extension(reference_root: str, force: bool = False) -> str:
    """Compile the reference extension (sm_100) into oracle/_ref/ca_ref_cuda.so."""
    cpp, cu, path = _source_strings(reference_root)
    if not force and os.path.exists(SO_PATH) and os.path.getmtime(SO_PATH) >= os.path.getmtime(path):
        return SO_PATH
    from torch.utils.cpp_extension import load_inline
    os.makedirs(REF_DIR, exist_ok=True)
    old_arch = os.environ.get("TORCH_CUDA_ARCH_LIST")
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0"
    tmp = tempfile.mkdtemp(prefix="ca_ref_cuda_")
    try:
        # the reference's own flags (cuda/continuum_attention.py:614-620)
        load_inline(name=MODULE_NAME, cpp_sources=cpp, cuda_sources=cu, functions=None, with_cuda=True,
                    extra_cflags=["-O2"], extra_cuda_cflags=["-O3"], build_directory=tmp, verbose=False)
        built = glob.glob(os.path.join(tmp, MODULE_NAME + "*.so"))
        if not built:
            raise RuntimeError("reference extension build produced no module")
        shutil.copy2(built[0], SO_PATH)
    finally:
        if old_arch is None:
            os.environ.pop("TORCH_CUDA_ARCH_LIST", None)
        else:
            os.environ["TORCH_CUDA_ARCH_LIST"] = old_arch
        shutil.rmtree(tmp, ignore_errors=True)
    return SO_PATH


_EXT = None


def available() -> bool:
    return os.path.exists(SO_PATH)


def extension():
    """The compiled reference extension module (import torch first)."""
    global _EXT
    if _EXT is None:
        if not available():
            raise RuntimeError(f"{SO_PATH} is not built")
        loader = importlib.machinery.ExtensionFileLoader(MODULE_NAME, SO_PATH)
        spec = importlib.util.spec_from_file_location(MODULE_NAME, SO_PATH, loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        _EXT = mod
    return _EXT


class RefTiledCA(torch.autograd.Function):
    """_CAExactTiled (cuda/continuum_attention.py:650-766) for modes prefix_v6 and prefix."""

    @staticmethod
    def forward(ctx, q, k, v, log_gain, query_tile, mode):
        ext = extension()
        B, H, T, D = q.shape
        if mode == "prefix_v6" and (q.dtype != torch.float16 or T > 2048):
            raise ValueError("prefix_v6 needs fp16 inputs and T <= 2048")
        scale = (log_gain.detach().exp().float() * D ** -0.5).reshape(H).contiguous()
        qb, kb, vb = (t.reshape(B * H, T, D) for t in (q, k, v))
        out = []
        for start in range(0, T, query_tile):
            end = min(T, start + query_tile)
            raw = torch.bmm(qb[:, start:end], kb[:, :end].transpose(1, 2))
            if mode == "prefix_v6":
                s = ext.scale_scores_half(raw.contiguous(), scale)
                w = ext.forward_half(s, start)
                y = torch.bmm(w, vb[:, :end])
            else:
                s = (raw.float().reshape(B, H, -1, end) * scale.view(1, H, 1, 1)).reshape(B * H, -1, end).contiguous()
                w = ext.forward(s, start)[0]
                y = torch.bmm(w.to(v.dtype), vb[:, :end])
            out.append(y)
        ctx.save_for_backward(q, k, v, log_gain)
        ctx.query_tile = int(query_tile)
        ctx.mode = mode
        return torch.cat(out, dim=1).reshape(B, H, T, D)

    @staticmethod
    def backward(ctx, grad_y):
        ext = extension()
        q, k, v, log_gain = ctx.saved_tensors
        B, H, T, D = q.shape
        scale = (log_gain.detach().exp().float() * D ** -0.5).reshape(H).contiguous()
        qb, kb, vb = (t.reshape(B * H, T, D) for t in (q, k, v))
        gb = grad_y.contiguous().reshape(B * H, T, D)
        gq = torch.zeros(B * H, T, D, device=q.device, dtype=torch.float32)
        gk = torch.zeros_like(gq)
        gv = torch.zeros_like(gq)
        gr = torch.zeros(H, device=q.device, dtype=torch.float32)
        for start in range(0, T, ctx.query_tile):
            end = min(T, start + ctx.query_tile)
            qs, keys, vals, gys = qb[:, start:end], kb[:, :end], vb[:, :end], gb[:, start:end]
            raw = torch.bmm(qs, keys.transpose(1, 2))
            if ctx.mode == "prefix_v6":
                s = ext.scale_scores_half(raw.contiguous(), scale)
                gw_half = torch.bmm(gys, vals.transpose(1, 2))
                w, ds_scaled, gain_rows = ext.backward_half_gw16(s, gw_half.contiguous(), scale, start)
                gv[:, :end].add_(torch.bmm(w.transpose(1, 2), gys).float())
                gq[:, start:end].add_(torch.bmm(ds_scaled, keys).float())
                gk[:, :end].add_(torch.bmm(ds_scaled.transpose(1, 2), qs).float())
                gr.add_(gain_rows.reshape(B, H, -1).sum(dim=(0, 2)))
            else:
                s = (raw.float().reshape(B, H, -1, end) * scale.view(1, H, 1, 1)).reshape(B * H, -1, end).contiguous()
                gw = torch.bmm(gys, vals.transpose(1, 2)).float().contiguous()
                w, ds = ext.backward_fused(s, gw, start)
                gv[:, :end].add_(torch.bmm(w.to(v.dtype).transpose(1, 2), gys).float())
                ds4 = ds.reshape(B, H, -1, end)
                scaled = (ds4 * scale.view(1, H, 1, 1)).reshape(B * H, -1, end)
                gq[:, start:end].add_(torch.bmm(scaled.to(q.dtype), keys).float())
                gk[:, :end].add_(torch.bmm(scaled.to(k.dtype).transpose(1, 2), qs).float())
                gr.add_((ds4 * s.reshape(B, H, -1, end)).sum(dim=(0, 2, 3)))
        return (gq.reshape_as(q).to(q.dtype), gk.reshape_as(k).to(k.dtype), gv.reshape_as(v).to(v.dtype),
                gr.to(log_gain.dtype), None, None)


def ref_continuum_attention(q, k, v, log_gain, query_tile=128, mode="prefix_v6"):
    """The reference op in one of its CUDA modes (inputs contiguous, as its wrapper makes them)."""
    return RefTiledCA.apply(q.contiguous(), k.contiguous(), v.contiguous(), log_gain, query_tile, mode)


if __name__ == "__main__":
    import argparse
    p = argparse.ArgumentParser(description="build oracle/_ref/ca_ref_cuda.so from the reference sources")
    p.add_argument("--reference", required=True, help="root of the reference project")
    p.add_argument("--force", action="store_true")
    a = p.parse_args()
    print(build_extension(a.reference, force=a.force))
