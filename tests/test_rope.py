"""qk-norm + 3D RoPE: oracle vs the reference's own CPU modules (golden
fixtures), and the in-place CUDA kernel (through the C ABI) vs the oracle."""
import numpy as np
import pytest
import torch

from oracle import blocks_ref as B
from oracle import nvfp4_ref as R
from tests.golden_util import load_golden


def test_oracle_tables_match_reference_rotary_module():
    g = load_golden("blocks_golden.npz")
    cos, sin = B.rope_tables(g["rope_pos"], (16, 16, 16))
    assert np.max(np.abs(cos - g["rope_cos"])) < 1e-5
    assert np.max(np.abs(sin - g["rope_sin"])) < 1e-5


def test_product_tables_match_reference_rotary_module():
    from h3_engine_b200.rope import reference_dims, rope_tables
    g = load_golden("blocks_golden.npz")
    cos, sin = rope_tables(torch.from_numpy(g["rope_pos"]), reference_dims(8))
    assert torch.equal(cos, torch.from_numpy(g["rope_cos"]))
    assert torch.equal(sin, torch.from_numpy(g["rope_sin"]))


def test_oracle_norm_rope_matches_reference_golden():
    g = load_golden("blocks_golden.npz")
    q = R.bf16_from_bits(g["rope_q_bits"])[0]                # [T, H, D]
    w = R.bf16_from_bits(g["rope_w_bits"])
    y = B.qk_norm_rope(q, w, 1e-5, g["rope_cos"], g["rope_sin"])
    for key in ("rope_fused_bits", "rope_split_bits"):
        ref = R.bf16_from_bits(g[key])[0]
        assert R.max_rel_err(y, ref) <= 1e-2
        # the reference rounds after each bf16 op; the oracle once
        assert np.mean(R.bf16_bits(y) != g[key][0]) < 0.25


def _run_kernel(cuda, q, k, v, wq, wk, eps, cos, sin):
    """Packs q|k|v into one [T, 3*H*D] buffer, runs the kernel in place."""
    from h3_engine_b200 import ops
    T, H, D = q.shape
    qkv = torch.cat([q.reshape(T, -1), k.reshape(T, -1), v.reshape(T, -1)], dim=1)
    qkv = qkv.to(torch.bfloat16).to(cuda).contiguous()
    ops.qk_norm_rope(qkv, H, D, q_off=0, k_off=H * D, wq=None if wq is None else wq.to(cuda),
                     wk=None if wk is None else wk.to(cuda), eps=eps,
                     cos=None if cos is None else cos.to(cuda),
                     sin=None if sin is None else sin.to(cuda))
    torch.cuda.synchronize()
    out = qkv.float().cpu().numpy()
    return out[:, :H * D].reshape(T, H, D), out[:, H * D:2 * H * D].reshape(T, H, D), \
        out[:, 2 * H * D:].reshape(T, H, D)


def _check(got, ref):
    # one bf16 rounding each side, fp32 vs fp64 math: within 2 bf16 ulp
    ulp = np.maximum(np.abs(ref), 1e-30) * 2.0 ** -7
    assert np.all(np.abs(got - ref) <= 2 * ulp + 1e-6)


@pytest.mark.gpu
def test_kernel_reference_layout_with_passthrough(cuda):
    """Reference convention: rope_freq_dim 8 -> 48 rotary dims of 64, 16 pass through."""
    g = load_golden("blocks_golden.npz")
    q = torch.from_numpy(R.bf16_from_bits(g["rope_q_bits"])[0].copy())
    w = torch.from_numpy(R.bf16_from_bits(g["rope_w_bits"]).copy()).to(torch.bfloat16)
    gen = torch.Generator().manual_seed(3)
    k = torch.randn(q.shape, generator=gen).to(torch.bfloat16).float()
    v = torch.randn(q.shape, generator=gen).to(torch.bfloat16).float()
    cos, sin = torch.from_numpy(g["rope_cos"]), torch.from_numpy(g["rope_sin"])
    gq, gk, gv = _run_kernel(cuda, q, k, v, w, w, 1e-5, cos, sin)
    _check(gq, B.qk_norm_rope(q.numpy(), w.float().numpy(), 1e-5, cos.numpy(), sin.numpy()))
    _check(gk, B.qk_norm_rope(k.numpy(), w.float().numpy(), 1e-5, cos.numpy(), sin.numpy()))
    assert np.array_equal(gv, v.numpy())                      # v untouched
    ref = R.bf16_from_bits(g["rope_fused_bits"])[0]
    assert R.max_rel_err(gq, ref) <= 1e-2                      # the reference's own output


@pytest.mark.gpu
def test_kernel_3d_rope_44_42_42(cuda):
    """24 heads x 128, RoPE 44/42/42 over (t, h, w), theta 1e4; a slice of the
    packed video grid (21x30x52) followed by audio tokens on 1-D positions."""
    from h3_engine_b200.rope import packed_positions, rope_tables
    pos = packed_positions((21, 30, 52), 1024)
    rows = torch.cat([torch.arange(0, 200), torch.arange(32700, 32760 + 64)])
    pos = pos[rows]
    cos, sin = rope_tables(pos, (44, 42, 42), 1e4)
    ocos, osin = B.rope_tables(pos.numpy(), (44, 42, 42), 1e4)
    assert np.max(np.abs(cos.numpy() - ocos)) < 1e-3           # fp32 angles up to ~40 rad
    T, H, D = rows.numel(), 24, 128
    gen = torch.Generator().manual_seed(4)
    q, k, v = (torch.randn(T, H, D, generator=gen).to(torch.bfloat16).float() for _ in range(3))
    wq = (1 + 0.1 * torch.randn(D, generator=gen)).to(torch.bfloat16)
    wk = (1 + 0.1 * torch.randn(D, generator=gen)).to(torch.bfloat16)
    gq, gk, gv = _run_kernel(cuda, q, k, v, wq, wk, 1e-6, cos, sin)
    _check(gq, B.qk_norm_rope(q.numpy(), wq.float().numpy(), 1e-6, cos.numpy(), sin.numpy()))
    _check(gk, B.qk_norm_rope(k.numpy(), wk.float().numpy(), 1e-6, cos.numpy(), sin.numpy()))
    assert np.array_equal(gv, v.numpy())


@pytest.mark.gpu
def test_kernel_norm_only_and_rope_only(cuda):
    gen = torch.Generator().manual_seed(5)
    T, H, D = 77, 4, 128
    q, k, v = (torch.randn(T, H, D, generator=gen).to(torch.bfloat16).float() for _ in range(3))
    w = (1 + 0.1 * torch.randn(D, generator=gen)).to(torch.bfloat16)
    gq, gk, _ = _run_kernel(cuda, q, k, v, w, w, 1e-6, None, None)
    _check(gq, B.qk_norm_rope(q.numpy(), w.float().numpy(), 1e-6))
    pos = torch.stack([torch.arange(T), torch.arange(T) % 7, torch.arange(T) % 5], 1).float()
    from h3_engine_b200.rope import rope_tables
    cos, sin = rope_tables(pos, (32, 32, 32))               # 96 rotary dims, 32 pass through
    gq, gk, _ = _run_kernel(cuda, q, k, v, None, None, 1e-6, cos, sin)
    _check(gk, B.qk_norm_rope(k.numpy(), None, 1e-6, cos.numpy(), sin.numpy()))
