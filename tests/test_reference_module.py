"""The reference's own ``H3TransformerBlock`` (h3_inference/transformer/model.py:157-209)
on this package, imported from a checkout of shauray8/h3-engine named by the
``H3_REFERENCE_ROOT`` environment variable.  The reference's source is not
part of this repository and does not travel with it, so every test here skips,
with that reason, where the variable is unset.

Two integration routes (the integration notes, section 1):

* ``module`` -- the model's kernel modules (``_ew``, ``_gemm``, ``_other``,
  ``_attn``, model.py:8-11) are this package's row shims;
* ``plugin`` -- the reference's own shims, unmodified, with their plug-in
  import (h3_inference/kernels/_dispatch.py:22-36) resolved to
  ``h3_engine_b200.kernels._dispatch``.

CPU: every row call of the block's forward reaches this package (counted as a
MISS: the kernels take no CPU tensors) and the stock expressions it then runs
reproduce the golden output of the reference's bf16 block bit for bit.
GPU: with ``H3_KERNELS=1`` every call takes a kernel (no MISS) and the block's
PSNR against the reference's bf16 output stays within 0.5 dB of the same
block with only its linears in NVFP4."""
import os
import sys
import types
from pathlib import Path

import numpy as np
import pytest
import torch
from torch import nn

from oracle import nvfp4_ref as R
from tests.golden_util import load_golden

FLAGS = ("H3_KERNELS", "H3_NVFP4", "H3_FUSED_ROPE", "H3_FUSED_MODULATE", "H3_TL_ATTN",
         "H3_FUSED_SWIGLU", "H3_FUSED_GATE")
TABLES = ["shift_msa", "scale_msa", "gate_msa", "shift_mlp", "scale_mlp", "gate_mlp"]


def _reference_root() -> Path:
    root = os.environ.get("H3_REFERENCE_ROOT")
    if not root:
        pytest.skip("H3_REFERENCE_ROOT is not set: the reference's source is not part of this "
                    "repository and is not present on this machine")
    root = Path(root)
    if not (root / "h3_inference" / "transformer" / "model.py").is_file():
        pytest.skip(f"no h3_inference/transformer/model.py under H3_REFERENCE_ROOT={root}")
    return root


@pytest.fixture
def reference(monkeypatch):
    """Imports ``h3_inference.transformer.model`` from the checkout; every
    module it added (and the plug-in alias) is dropped again afterwards."""
    root = _reference_root()
    for fl in FLAGS:
        monkeypatch.delenv(fl, raising=False)
    monkeypatch.setenv("H3_NO_MAIKU", "0")
    before = set(sys.modules)
    monkeypatch.syspath_prepend(str(root))
    import h3_inference.transformer.model as model
    import h3_inference.kernels._dispatch as ref_dispatch
    yield types.SimpleNamespace(model=model, dispatch=ref_dispatch)
    for name in set(sys.modules) - before:
        if name.startswith(("h3_inference", "maiku")):
            del sys.modules[name]


def _route(ref, route, monkeypatch):
    from h3_engine_b200.kernels import _dispatch
    from h3_engine_b200.kernels import elementwise_norm_rope as ew
    from h3_engine_b200.kernels import ffn_qkvo_gemms as gm
    from h3_engine_b200.kernels import other as ot
    from h3_engine_b200.kernels import packed_self_attn as at
    if route == "module":
        for name, mod in (("_ew", ew), ("_gemm", gm), ("_other", ot), ("_attn", at)):
            monkeypatch.setattr(ref.model, name, mod)
    else:
        pkg = types.ModuleType("maiku")
        pkg.dispatch = _dispatch
        monkeypatch.setitem(sys.modules, "maiku", pkg)
        monkeypatch.setitem(sys.modules, "maiku.dispatch", _dispatch)
        monkeypatch.setattr(ref.dispatch, "_maiku_state", "unloaded")
        monkeypatch.setattr(ref.dispatch, "_maiku_try_call", None)
    return _dispatch


def _golden_block(model, device):
    g = load_golden("refblock_golden.npz")
    C = g["x_bits"].shape[-1]
    heads, d = 2, 128
    f = g["w.ff.net.2.weight_bits"].shape[1]
    eps = float(g["eps"][0])
    blk = model.H3TransformerBlock(C, heads, d, f, time_embed_dim=64, norm_eps=eps,
                                   qk_norm_eps=eps)
    bf = lambda key: torch.from_numpy(R.bf16_from_bits(g[key]).astype(np.float32))  # noqa: E731
    with torch.no_grad():
        for name, p in blk.named_parameters():
            if not name.startswith("adaln_proj"):
                p.copy_(bf("w." + name + "_bits"))
    blk = blk.to(device).to(torch.bfloat16).eval()
    blk.folded_modulation = tuple(bf(n + "_bits").to(device).to(torch.bfloat16) for n in TABLES)
    x = bf("x_bits").to(device).to(torch.bfloat16)
    idx = torch.from_numpy(g["idx"]).to(device)
    cos, sin = (torch.from_numpy(g[k]).to(device) for k in ("cos", "sin"))
    return blk, (x, None, idx, (cos, sin)), g["y_bits"]


@pytest.mark.parametrize("route", ["module", "plugin"])
def test_reference_block_reaches_this_package_on_cpu(reference, route, monkeypatch):
    dispatch = _route(reference, route, monkeypatch)
    blk, args, y_bits = _golden_block(reference.model, "cpu")
    if route == "module":
        # armed: each row call reaches a shim here, which refuses CPU tensors
        # (MISS) and runs the reference's stock expression
        monkeypatch.setenv("H3_KERNELS", "1")
        expect = {"norm_modulate_h3", "norm_rope_h3", "gate_residual_gather",
                  "qkv_projection", "out_projection", "ffn", "attention"}
    else:
        # the reference's own shims, armed only where their MISS path is eager
        # (the others compile their expression); every plug-in call is
        # answered (MISS) by this package's try_call
        for fl in ("H3_NVFP4", "H3_TL_ATTN"):
            monkeypatch.setenv(fl, "1")
        expect = {"qkv_projection", "out_projection", "ffn", "attention"}
    dispatch.miss_counts(reset=True)
    with torch.no_grad():
        y = blk(*args)
    misses = dispatch.miss_counts()
    assert expect <= set(misses), sorted(misses.items())
    assert np.array_equal(R.bf16_bits(y.float().numpy()), y_bits)


def _psnr(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return 10 * np.log10(np.max(np.abs(ref)) ** 2 / np.mean((got - ref) ** 2))


@pytest.mark.gpu
@pytest.mark.parametrize("route", ["module", "plugin"])
def test_reference_block_on_the_kernels(reference, route, cuda, monkeypatch):
    from h3_engine_b200 import nvfp4
    dispatch = _route(reference, route, monkeypatch)
    blk, args, y_bits = _golden_block(reference.model, cuda)

    class _Model(nn.Module):
        def __init__(self, b):
            super().__init__()
            self.transformer_blocks = nn.ModuleList([b])
    stats = nvfp4.quantize_blocks(_Model(blk), self_check=False)
    assert stats["linears_quantized"] == 6
    y_ref = R.bf16_from_bits(y_bits)
    with torch.no_grad():
        y_stock = blk(*args)                 # NVFP4 linears, stock torch elsewhere
    monkeypatch.setenv("H3_KERNELS", "1")
    dispatch.miss_counts(reset=True)
    with torch.no_grad():
        y = blk(*args)
    torch.cuda.synchronize()
    assert dispatch.miss_counts() == {}     # every armed call took a kernel
    p_kern = _psnr(y.float().cpu().numpy(), y_ref)
    p_stock = _psnr(y_stock.float().cpu().numpy(), y_ref)
    assert p_kern >= p_stock - 0.5, (p_kern, p_stock)
