"""Regenerate the committed golden fixtures in this folder.

    python tests/golden/make_golden.py --reference /path/to/h3-engine

Run in a container where the reference checkout is present (it is read, never
modified).  What comes from where:

* ``nvfp4_golden.npz`` -- inputs and the CPU oracle's packed bytes / scales /
  global scale for seeded cases and hand-made edge cases (a regression pin of
  the recipe), plus the reference's OWN decode of two-level packed weights:
  ``h3_inference/render.py:_Fp4Linear.forward`` (``:174-183``, LUT ``:185-188``)
  run on CPU.  That method reads one constant from the absent ``maiku``
  package, so a stub module supplies it; the decode itself is the reference's.
* ``blocks_golden.npz`` -- the reference's stock CPU modules at small shapes:
  ``nn.RMSNorm``, ``_norm_rope_impl`` / ``apply_rotary_emb``
  (``h3_inference/kernels/elementwise_norm_rope.py:25-40,104-122``),
  ``H3RotaryPosEmbed`` (``h3_inference/transformer/model.py:23-38``) and
  ``packed_self_attention`` (SDPA path, ``h3_inference/kernels/packed_self_attn.py:31-37``).
* ``refblock_golden.npz`` -- one ``H3TransformerBlock`` of the reference model
  (``h3_inference/transformer/model.py:157-209``: RMSNorm + gather-modulate,
  attention with qk-norm and 16/16/16 RoPE, gated residual, SwiGLU
  feed-forward) run in bf16 on CPU through its stock paths, at small shapes
  (hidden 256, 2 heads x 128, ffn 256, 128 tokens, three modality tables).
"""
from __future__ import annotations

import argparse
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import nvfp4_ref as R  # noqa: E402


def _rng(seed: int) -> torch.Generator:
    return torch.Generator(device="cpu").manual_seed(seed)


def bf16_randn(shape, seed: int, std: float = 1.0, outlier_frac: float = 0.0) -> np.ndarray:
    g = _rng(seed)
    x = torch.randn(*shape, generator=g, dtype=torch.float32) * std
    if outlier_frac:
        n = x.numel()
        idx = torch.randperm(n, generator=g)[: max(1, int(n * outlier_frac))]
        x.view(-1)[idx] *= 50.0
    return x.to(torch.bfloat16).float().numpy()


def edge_case_matrix() -> np.ndarray:
    """Rows exercising the recipe's corners (K = 64 -> 4 blocks per row)."""
    K = 64
    rows = []
    rows.append(np.zeros(K))                                   # all-zero row
    r = np.zeros(K); r[:16] = -0.0; r[16:32] = 1e-30; rows.append(r)   # -0, tiny
    # exact E2M1 midpoints once the block scale is 1 (bmax = 6 * d6): ties
    r = np.tile(np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0]), 8).astype(np.float64)
    rows.append(r)
    rows.append(-r)
    r = np.linspace(-448 * 6, 448 * 6, K); rows.append(r)     # spans the global range
    r = np.full(K, 3.0e-6); r[::2] *= -1; rows.append(r)      # tiny block vs large amax
    r = np.zeros(K); r[5] = 7.0; r[40] = -1e-3; rows.append(r)  # one nonzero per block
    r = np.arange(K, dtype=np.float64) - 31.5; rows.append(r)
    m = np.stack(rows).astype(np.float32)
    return R.bf16_round(m)


def nvfp4_cases(ref_root: Path) -> dict[str, np.ndarray]:
    out: dict[str, np.ndarray] = {}
    cases = {
        "randn": bf16_randn((256, 512), seed=1, outlier_frac=0.001),
        "ragged": bf16_randn((77, 192), seed=5),
        "edge": edge_case_matrix(),
        "weight": bf16_randn((128, 256), seed=0, std=0.02),
    }
    for name, x in cases.items():
        q, sf, gs = R.quantize(x, mpad=R.pad_m(x.shape[0]))
        out[f"{name}_x_bits"] = R.bf16_bits(x)
        out[f"{name}_q"] = q
        out[f"{name}_sf"] = sf
        out[f"{name}_sf_swizzled"] = R.swizzle(sf)
        out[f"{name}_gs"] = np.array([gs], dtype=np.float32)
        out[f"{name}_deq_bits"] = R.bf16_bits(R.dequantize(q, sf, gs)[: x.shape[0]])

    # The reference's own CPU decode of two-level (gs = 1) packed weights.
    sys.path.insert(0, str(ref_root))
    stub = types.ModuleType("maiku.kernels.quant.nvfp4")
    stub._B = R.FP4_BLOCK
    for mod in ("maiku", "maiku.kernels", "maiku.kernels.quant"):
        sys.modules.setdefault(mod, types.ModuleType(mod))
    sys.modules["maiku.kernels.quant.nvfp4"] = stub
    from h3_inference import render as ref_render

    w = cases["weight"]
    q2, sf2, _ = R.quantize(w, gs=1.0)
    lin = ref_render._Fp4Linear.__new__(ref_render._Fp4Linear)
    torch.nn.Module.__init__(lin)
    lin.register_buffer("qdata", torch.from_numpy(q2.copy()))
    lin.register_buffer("scale", torch.from_numpy(sf2.copy()).view(torch.float8_e4m3fn))
    lin.block = R.FP4_BLOCK
    lin.bias = None
    lin.out_features, lin.in_features = w.shape
    lin.orig_dtype = torch.bfloat16
    eye = torch.eye(w.shape[1], dtype=torch.float32)
    with torch.no_grad():
        deq_ref = lin(eye).T.contiguous().numpy()     # [N, K]: the reference's decoded weight
    out["ref2_q"] = q2
    out["ref2_sf"] = sf2
    out["ref2_deq_f32"] = deq_ref.astype(np.float32)
    out["ref2_lut"] = ref_render._E2M1_LUT.numpy()
    return out


def block_cases(ref_root: Path) -> dict[str, np.ndarray]:
    sys.path.insert(0, str(ref_root))
    from h3_inference.kernels import elementwise_norm_rope as ew
    from h3_inference.kernels import packed_self_attn as psa
    from h3_inference.transformer.model import H3RotaryPosEmbed

    out: dict[str, np.ndarray] = {}
    g = _rng(7)
    T, H, D, hidden = 48, 4, 64, 256
    x = torch.randn(1, T, hidden, generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(hidden, generator=g)).to(torch.bfloat16)
    norm = torch.nn.RMSNorm(hidden, eps=1e-6).to(torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(gamma)
        y = ew.rms_norm(norm, x)
    out["rms_x_bits"] = R.bf16_bits(x.float().numpy())
    out["rms_gamma_bits"] = R.bf16_bits(gamma.float().numpy())
    out["rms_y_bits"] = R.bf16_bits(y.float().numpy())
    out["rms_eps"] = np.array([1e-6], dtype=np.float32)

    # reference-convention 3-axis RoPE: rope_freq_dim 8 -> 48 rotary dims of 64
    rope = H3RotaryPosEmbed(rope_freq_dim=8, rope_theta=10000.0)
    pos = torch.stack([torch.arange(T) // 12, (torch.arange(T) // 4) % 3, torch.arange(T) % 4],
                      dim=1).float()
    cos, sin = rope(pos)
    q = torch.randn(1, T, H, D, generator=g).to(torch.bfloat16)
    qn = torch.nn.RMSNorm(D, eps=1e-5).to(torch.bfloat16)
    with torch.no_grad():
        qn.weight.copy_((1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16))
        y_fused = ew._norm_rope_impl(q, qn.weight, 1e-5, cos, sin)
        y_split = ew.apply_rotary_emb(ew.qk_norm(qn, q), cos, sin)
    out["rope_pos"] = pos.numpy()
    out["rope_cos"] = cos.numpy()
    out["rope_sin"] = sin.numpy()
    out["rope_q_bits"] = R.bf16_bits(q.float().numpy())
    out["rope_w_bits"] = R.bf16_bits(qn.weight.detach().float().numpy())
    out["rope_fused_bits"] = R.bf16_bits(y_fused.float().numpy())
    out["rope_split_bits"] = R.bf16_bits(y_split.float().numpy())

    qa = torch.randn(1, T, H, D, generator=g).to(torch.bfloat16)
    ka = torch.randn(1, T, H, D, generator=g).to(torch.bfloat16)
    va = torch.randn(1, T, H, D, generator=g).to(torch.bfloat16)
    with torch.no_grad():
        oa = psa.packed_self_attention(qa.float(), ka.float(), va.float(), None)
    out["attn_q_bits"] = R.bf16_bits(qa.float().numpy())
    out["attn_k_bits"] = R.bf16_bits(ka.float().numpy())
    out["attn_v_bits"] = R.bf16_bits(va.float().numpy())
    out["attn_o_f32"] = oa.numpy().astype(np.float32)
    return out


def ref_block_case(ref_root: Path) -> dict[str, np.ndarray]:
    sys.path.insert(0, str(ref_root))
    from h3_inference.transformer.model import H3RotaryPosEmbed, H3TransformerBlock

    C, H, D, F, T = 256, 2, 128, 256, 128
    g = _rng(21)
    blk = H3TransformerBlock(C, H, D, F, time_embed_dim=64, norm_eps=1e-5, qk_norm_eps=1e-5)
    blk = blk.to(torch.bfloat16).eval()
    with torch.no_grad():
        for name, p in blk.named_parameters():
            if name.endswith("norm1.weight") or name.endswith("norm2.weight") or "norm_q" in name \
                    or "norm_k" in name:
                p.copy_(1 + 0.1 * torch.randn(p.shape, generator=g))
            elif p.dim() == 2:
                p.copy_(torch.randn(p.shape, generator=g) / p.shape[1] ** 0.5)
            else:
                p.copy_(0.01 * torch.randn(p.shape, generator=g))
        tables = [0.1 * torch.randn(3, C, generator=g) for _ in range(2)]
        tables.append(0.5 + 0.2 * torch.randn(3, C, generator=g))           # gate_msa
        tables += [0.1 * torch.randn(3, C, generator=g) for _ in range(2)]
        tables.append(0.5 + 0.2 * torch.randn(3, C, generator=g))           # gate_mlp
        tables = [t.to(torch.bfloat16) for t in tables]
        blk.folded_modulation = tuple(tables)
        x = torch.randn(1, T, C, generator=g).to(torch.bfloat16)
        idx = torch.cat([torch.zeros(96), torch.ones(16), 2 * torch.ones(16)]).long()
        pos = torch.stack([torch.arange(T) // 32, (torch.arange(T) // 8) % 4,
                           torch.arange(T) % 8], dim=1).float()
        cos, sin = H3RotaryPosEmbed(rope_freq_dim=16, rope_theta=10000.0)(pos)
        y = blk(x, None, idx, (cos, sin))
    out = {"x_bits": R.bf16_bits(x.float().numpy()), "y_bits": R.bf16_bits(y.float().numpy()),
           "idx": idx.numpy(), "pos": pos.numpy(), "cos": cos.numpy(), "sin": sin.numpy(),
           "eps": np.array([1e-5], dtype=np.float32)}
    names = ["shift_msa", "scale_msa", "gate_msa", "shift_mlp", "scale_mlp", "gate_mlp"]
    for n, t in zip(names, tables):
        out[n + "_bits"] = R.bf16_bits(t.float().numpy())
    for name, p in blk.named_parameters():
        if name.startswith("adaln_proj"):
            continue
        out["w." + name + "_bits"] = R.bf16_bits(p.detach().float().numpy())
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("H3_REFERENCE_ROOT"),
                    help="checkout of shauray8/h3-engine (or set H3_REFERENCE_ROOT)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set H3_REFERENCE_ROOT to the reference checkout")
    ref_root = Path(args.reference)
    np.savez_compressed(HERE / "nvfp4_golden.npz", **nvfp4_cases(ref_root))
    np.savez_compressed(HERE / "blocks_golden.npz", **block_cases(ref_root))
    np.savez_compressed(HERE / "refblock_golden.npz", **ref_block_case(ref_root))
    print("wrote", HERE / "nvfp4_golden.npz", HERE / "blocks_golden.npz",
          HERE / "refblock_golden.npz")


if __name__ == "__main__":
    main()
