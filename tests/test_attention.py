"""Packed varlen attention: oracle vs the reference's own SDPA path (golden
fixture), and the tcgen05 kernel (through the C ABI) vs the oracle and vs
torch's scaled_dot_product_attention run per document on the same inputs.

Tolerance: max|o - ref| / max|ref| <= 1e-2 (bf16 in/out, fp32 softmax)."""
import numpy as np
import pytest
import torch

from oracle import blocks_ref as B
from oracle import nvfp4_ref as R
from tests.golden_util import load_golden

TOL = 1e-2


def test_oracle_matches_reference_sdpa_golden():
    g = load_golden("blocks_golden.npz")
    q = R.bf16_from_bits(g["attn_q_bits"])[0]
    k = R.bf16_from_bits(g["attn_k_bits"])[0]
    v = R.bf16_from_bits(g["attn_v_bits"])[0]
    o = B.attention(q, k, v, [0, q.shape[0]])
    assert np.max(np.abs(o - g["attn_o_f32"][0])) < 1e-5


def _qkv(T, H, D, seed, spread=1.0):
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(T, H, D, generator=g) * spread for _ in range(3))
    return [t.to(torch.bfloat16) for t in (q, k, v)]


def _run(cuda, q, k, v, cu):
    from h3_engine_b200 import ops
    T, H, D = q.shape
    qkv = torch.cat([q.reshape(T, -1), k.reshape(T, -1), v.reshape(T, -1)], 1).to(cuda).contiguous()
    o = ops.attention_varlen(qkv, H, D, cu, q_off=0, k_off=H * D, v_off=2 * H * D)
    torch.cuda.synchronize()
    return o.float().cpu().numpy().reshape(T, H, D), qkv


def _cu(lens):
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    return cu


# 64 documents (the kernel's maximum): empty, single-token, tile-edge
# (127/128/129, 255/256/257) and ragged lengths
RAGGED = _cu([0, 1, 2, 127, 128, 129, 255, 256, 257, 3, 64, 0, 5, 1]
             + [17 * (i % 9) + 1 for i in range(50)])


@pytest.mark.gpu
@pytest.mark.parametrize("cu,H", [([0, 128], 1), ([0, 300, 700], 2), ([0, 1000, 1050, 1300], 3),
                                  ([0, 2048], 4), (RAGGED, 2)])
def test_kernel_matches_oracle(cuda, cu, H):
    T, D = cu[-1], 128
    q, k, v = _qkv(T, H, D, seed=len(cu) + H)
    o, _ = _run(cuda, q, k, v, cu)
    ref = B.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), cu)
    assert np.isfinite(o).all()
    assert R.max_rel_err(o, ref) <= TOL


@pytest.mark.gpu
def test_kernel_sharp_scores_rescaling(cuda):
    """Large logits make the running row max grow across key tiles (exercises
    the in-TMEM rescale of O)."""
    cu = [0, 1024]
    q, k, v = _qkv(1024, 2, 128, seed=9, spread=3.0)
    o, _ = _run(cuda, q, k, v, cu)
    ref = B.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), cu)
    assert R.max_rel_err(o, ref) <= TOL


@pytest.mark.gpu
def test_kernel_agrees_with_torch_sdpa(cuda):
    """The reference's attention call (F.scaled_dot_product_attention) per document."""
    import torch.nn.functional as F
    cu = [0, 640, 900]
    q, k, v = _qkv(900, 4, 128, seed=11)
    o, _ = _run(cuda, q, k, v, cu)
    ref = []
    for a, b in zip(cu[:-1], cu[1:]):
        qs, ks, vs = (t[a:b].to(cuda).transpose(0, 1)[None] for t in (q, k, v))
        ref.append(F.scaled_dot_product_attention(qs, ks, vs)[0].transpose(0, 1))
    ref = torch.cat(ref).float().cpu().numpy()
    assert R.max_rel_err(o, ref) <= TOL


@pytest.mark.gpu
def test_kernel_packed_video_audio_full_size_row_sample(cuda):
    """The configured packing: 32760 video tokens + 1024 audio tokens, 24 heads x 128,
    documents [0, 32760, 33784]; a query-row sample through the oracle."""
    cu = [0, 32760, 33784]
    T, H, D = 33784, 24, 128
    g = torch.Generator(device=cuda).manual_seed(3)
    qkv = torch.randn(T, 3 * H * D, generator=g, device=cuda).to(torch.bfloat16)
    from h3_engine_b200 import ops
    o = ops.attention_varlen(qkv, H, D, cu, q_off=0, k_off=H * D, v_off=2 * H * D)
    rows = np.concatenate([np.arange(0, 8), np.arange(32750, 32770), np.arange(33776, 33784),
                           np.random.default_rng(0).integers(0, T, 24)])
    x = qkv.float().cpu().numpy().reshape(T, 3, H, D)
    ref = B.attention(x[:, 0], x[:, 1], x[:, 2], cu, rows=rows)
    got = o.float().cpu().numpy().reshape(T, H, D)[rows]
    assert R.max_rel_err(got, ref) <= TOL


@pytest.mark.gpu
def test_token_sharded_queries_match_unsharded(cuda):
    """Sequence parallelism: each shard's query rows against the gathered
    keys / values give exactly the unsharded rows (same key tiles, same order)."""
    from h3_engine_b200 import ops
    cu = [0, 700, 1000, 1500]
    T, H, D = 1500, 2, 128
    q, k, v = _qkv(T, H, D, seed=13)
    full, qkv = _run(cuda, q, k, v, cu)
    parts = []
    for a, b in [(0, 350), (350, 1100), (1100, 1500)]:
        o = ops.attention_varlen(qkv[a:b], H, D, cu, q_off=0, k_off=H * D, v_off=2 * H * D,
                                 kv=qkv, q_row0=a)
        parts.append(o)
    got = torch.cat(parts).float().cpu().numpy().reshape(T, H, D)
    assert np.array_equal(got, full)
