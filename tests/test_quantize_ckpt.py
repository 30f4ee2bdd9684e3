"""Packed-checkpoint writer and loader round trip on the GPU: a small two-shard
bf16 checkpoint of two transformer blocks is quantized by
``h3_engine_b200.quantize_ckpt.run`` (the drop-in for
h3_inference/quantize_ckpt.py), checked byte for byte against the oracle,
then loaded into a block-shaped model by ``nvfp4.load_quantized`` and run."""
import json

import numpy as np
import pytest
import torch
from torch import nn

from oracle import nvfp4_ref as R

D, F = 256, 512


class _GeluProj(nn.Module):
    def __init__(self):
        super().__init__()
        self.proj = nn.Linear(D, F, bias=False)


class _Attn(nn.Module):
    def __init__(self):
        super().__init__()
        self.to_q = nn.Linear(D, D, bias=False)
        self.to_k = nn.Linear(D, D, bias=False)
        self.to_v = nn.Linear(D, D, bias=False)
        self.to_out = nn.ModuleList([nn.Linear(D, D, bias=False), nn.Dropout(0.0)])


class _FF(nn.Module):
    def __init__(self):
        super().__init__()
        self.net = nn.ModuleList([_GeluProj(), nn.Dropout(0.0), nn.Linear(F, D, bias=False)])


class _Block(nn.Module):
    def __init__(self):
        super().__init__()
        self.attn = _Attn()
        self.ff = _FF()
        self.norm1 = nn.LayerNorm(D)


class _Model(nn.Module):
    def __init__(self, blocks=2):
        super().__init__()
        self.transformer_blocks = nn.ModuleList([_Block() for _ in range(blocks)])
        self.proj_out = nn.Linear(D, D, bias=False)


def _checkpoint(tmp_path):
    from safetensors.torch import save_file
    torch.manual_seed(11)
    model = _Model().to(torch.bfloat16)
    with torch.no_grad():
        for p in model.parameters():
            p.copy_(torch.randn_like(p) * 0.02)
    sd = {k: v.contiguous() for k, v in model.state_dict().items()}
    keys = sorted(sd)
    half = len(keys) // 2
    src = tmp_path / "bf16"
    src.mkdir()
    shards = {"a.safetensors": keys[:half], "b.safetensors": keys[half:]}
    wm = {}
    for name, ks in shards.items():
        save_file({k: sd[k] for k in ks}, str(src / name))
        wm.update({k: name for k in ks})
    (src / "model.safetensors.index.json").write_text(json.dumps({"weight_map": wm}))
    (src / "config.json").write_text(json.dumps({"hidden": D}))
    return model, sd, src


@pytest.mark.gpu
def test_quantize_checkpoint_roundtrip(cuda, tmp_path):
    from safetensors import safe_open
    from h3_engine_b200 import nvfp4, quantize_ckpt

    model, sd, src = _checkpoint(tmp_path)
    dst = tmp_path / "nvfp4"
    assert quantize_ckpt.run(str(src), str(dst), verify=True, log=lambda *_: None) == 0
    index = json.loads((dst / "model.safetensors.index.json").read_text())
    assert index["metadata"]["h3_quant"] == "nvfp4"
    assert (dst / "config.json").exists()
    wm = index["weight_map"]
    quantizable = [k for k in sd if quantize_ckpt.is_quantizable(k)]
    assert len(quantizable) == 12                          # 6 linears x 2 blocks
    for k in sd:
        if k in quantizable:
            assert k not in wm and k + "_nvfp4" in wm and k + "_nvfp4_scale" in wm
        else:
            assert k in wm                                 # copied through
    # bytes of every quantized weight equal the oracle's
    for k in quantizable:
        with safe_open(str(dst / wm[k + "_nvfp4"]), framework="pt") as f:
            q = f.get_tensor(k + "_nvfp4").numpy()
        with safe_open(str(dst / wm[k + "_nvfp4_scale"]), framework="pt") as f:
            sc = f.get_tensor(k + "_nvfp4_scale").numpy()
        with safe_open(str(dst / wm[k + "_nvfp4_global_scale"]), framework="pt") as f:
            gs = f.get_tensor(k + "_nvfp4_global_scale").numpy()
        w = sd[k].float().numpy()
        rq, rs, rgs = R.quantize(w)
        n, kk = w.shape
        assert np.array_equal(q, rq), k
        assert np.array_equal(R.unswizzle(sc, n, kk // 16), rs), k
        assert gs[0] == rgs, k
    # load into a fresh model and run one quantized linear against the oracle
    fresh = _Model().to(torch.bfloat16).to(cuda)
    summary = nvfp4.load_quantized(fresh, str(dst))
    assert summary["linears_loaded"] == 12
    lin = fresh.transformer_blocks[1].ff.net[0].proj
    assert isinstance(lin, nvfp4._QuantLinear)
    x = (torch.randn(64, D, generator=torch.Generator().manual_seed(3))).to(torch.bfloat16)
    y = lin(x.to(cuda)).float().cpu().numpy()
    w = sd["transformer_blocks.1.ff.net.0.proj.weight"].float().numpy()
    xq = R.quantize(x.float().numpy())
    ref = R.gemm_ref(*xq, *R.quantize(w), M=64, N=F)
    assert R.max_rel_err(y, ref) <= 1e-2


def test_is_quantizable_matches_reference_selection():
    from h3_engine_b200.quantize_ckpt import is_quantizable
    assert is_quantizable("transformer_blocks.3.attn.to_q.weight")
    assert is_quantizable("transformer_blocks.0.attn.to_out.0.weight")
    assert is_quantizable("transformer_blocks.47.ff.net.0.proj.weight")
    assert is_quantizable("transformer_blocks.1.ff.net.2.weight")
    assert not is_quantizable("transformer_blocks.1.attn.to_q.bias")
    assert not is_quantizable("transformer_blocks.1.norm1.weight")
    assert not is_quantizable("proj_out.weight")
