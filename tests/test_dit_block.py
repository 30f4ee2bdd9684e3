"""Attention sub-block and full DiT block (GPU, through the C ABI) vs the CPU
oracle; token-sharded execution vs unsharded.  Tolerance 1e-2 (max rel)."""
import numpy as np
import pytest
import torch

from oracle import blocks_ref as B
from oracle import nvfp4_ref as R

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _w(g, n, k, std=0.02):
    return (torch.randn(n, k, generator=g) * std).to(torch.bfloat16)


def make_attn(d, H, seed):
    g = torch.Generator().manual_seed(seed)
    HD = H * 128
    p = dict(wq=_w(g, HD, d), wk=_w(g, HD, d), wv=_w(g, HD, d), wo=_w(g, d, HD),
             gamma=(1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16),
             norm_q=(1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16),
             norm_k=(1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16))
    return p, g


def q3(w):
    return R.quantize(w.float().numpy())


def positions(T):
    return torch.stack([torch.arange(T) // 40, (torch.arange(T) // 8) % 5, torch.arange(T) % 8],
                       1).float()


def build_attn(p, H, cuda):
    from h3_engine_b200.blocks import AttnBlock
    return AttnBlock(p["wq"].to(cuda), p["wk"].to(cuda), p["wv"].to(cuda), p["wo"].to(cuda),
                     p["gamma"].to(cuda), p["norm_q"].to(cuda), p["norm_k"].to(cuda), H,
                     eps=1e-6, qk_eps=1e-6)


def test_attn_block_matches_oracle(cuda):
    from h3_engine_b200.rope import rope_tables
    T, d, H = 300, 512, 4
    cu = [0, 220, 300]
    p, g = make_attn(d, H, seed=1)
    x = torch.randn(T, d, generator=g).to(torch.bfloat16)
    cos, sin = rope_tables(positions(T), (44, 42, 42), 1e4)
    blk = build_attn(p, H, cuda)
    y = blk(x.to(cuda), (cos.to(cuda), sin.to(cuda)), cu).float().cpu().numpy()
    ref = B.attn_block(x.float().numpy(), p["gamma"].float().numpy(), 1e-6, q3(p["wq"]),
                       q3(p["wk"]), q3(p["wv"]), q3(p["wo"]), p["norm_q"].float().numpy(),
                       p["norm_k"].float().numpy(), 1e-6, H, cos.numpy(), sin.numpy(), cu)
    assert R.max_rel_err(y, ref) <= TOL


def test_dit_block_with_adaln_matches_oracle(cuda):
    from h3_engine_b200.blocks import DiTBlock, FFNBlock
    from h3_engine_b200.rope import rope_tables
    T, d, H, f = 256, 512, 4, 1024
    cu = [0, 256]
    p, g = make_attn(d, H, seed=2)
    w1, w2 = _w(g, f, d), _w(g, d, f)
    b1 = (0.01 * torch.randn(f, generator=g)).to(torch.bfloat16)
    b2 = (0.01 * torch.randn(d, generator=g)).to(torch.bfloat16)
    gamma2 = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    mod = [(0.1 * torch.randn(3, d, generator=g)).to(torch.bfloat16) for _ in range(6)]
    idx = torch.randint(0, 3, (T,), generator=g, dtype=torch.int32)
    x = torch.randn(T, d, generator=g).to(torch.bfloat16)
    cos, sin = rope_tables(positions(T), (44, 42, 42), 1e4)
    blk = DiTBlock(build_attn(p, H, cuda),
                   FFNBlock(w1.to(cuda), b1.to(cuda), w2.to(cuda), b2.to(cuda), gamma2.to(cuda)))
    y = blk(x.to(cuda), (cos.to(cuda), sin.to(cuda)), cu, tuple(m.to(cuda) for m in mod),
            idx.to(cuda)).float().cpu().numpy()
    m = [t.float().numpy() for t in mod]
    h = B.attn_block(x.float().numpy(), p["gamma"].float().numpy(), 1e-6, q3(p["wq"]),
                     q3(p["wk"]), q3(p["wv"]), q3(p["wo"]), p["norm_q"].float().numpy(),
                     p["norm_k"].float().numpy(), 1e-6, H, cos.numpy(), sin.numpy(), cu,
                     shift=m[0], scale=m[1], gate=m[2], mod_idx=idx.numpy())
    ref = B.ffn_block_mod(h, gamma2.float().numpy(), 1e-6, q3(w1), b1.float().numpy(), q3(w2),
                          b2.float().numpy(), shift=m[3], scale=m[4], gate=m[5],
                          mod_idx=idx.numpy())
    assert R.max_rel_err(y, ref) <= TOL


def test_sharded_attn_block_reproduces_unsharded(cuda):
    """Two token shards run one after the other on one GPU; their collectives
    replay the unsharded run (global amaxes, full K|V), so every output row
    must equal the unsharded one bit for bit."""
    from h3_engine_b200.blocks import SequenceShard
    from h3_engine_b200.rope import rope_tables
    T, d, H = 512, 512, 4
    HD = H * 128
    cu = [0, 384, 512]
    p, g = make_attn(d, H, seed=3)
    x = torch.randn(T, d, generator=g).to(torch.bfloat16).to(cuda)
    cos, sin = (t.to(cuda) for t in rope_tables(positions(T), (44, 42, 42), 1e4))
    blk = build_attn(p, H, cuda)
    full = blk(x, (cos, sin), cu).clone()
    ws = blk._ws[("attn", T, d, HD, x.device, False)]
    amax_norm = ws["norm"]["amax"].clone()
    amax_o = ws["amax_o"].clone()
    # the unsharded K|V per head group: [K heads of the group | V heads of it]
    G = blk._groups_for(None)
    hg = HD // G
    kv_groups = [torch.cat([ws["qkv"][:, HD + g * hg:HD + (g + 1) * hg],
                            ws["qkv"][:, 2 * HD + g * hg:2 * HD + (g + 1) * hg]], 1).clone()
                 for g in range(G)]
    for a, b in [(0, 256), (256, 512)]:
        seen = []

        def reduce_max(t):
            ref = amax_norm if not seen else amax_o
            assert t.item() <= ref.item()
            t.copy_(ref)
            seen.append(1)

        calls = []

        def all_gather(kv, local):
            # one call per head group, in order; the local K|V rows after
            # norm + RoPE equal the unsharded run's
            g = len(calls)
            calls.append(g)
            assert torch.equal(local, kv_groups[g][a:b])
            kv[:T].copy_(kv_groups[g])

        shard = SequenceShard(a, b - a, T, all_gather, reduce_max)
        y = blk(x[a:b], (cos[a:b], sin[a:b]), cu, shard=shard)
        torch.cuda.synchronize()
        assert calls == list(range(G)) and G == 2
        assert torch.equal(y, full[a:b])
