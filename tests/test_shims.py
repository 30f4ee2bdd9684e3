"""Row shims (``h3_engine_b200.kernels``, the reference's
``h3_inference/kernels`` surface): dispatch semantics and the SwiGLU weight
re-layout on the CPU; each flag-armed shim against the stock expression it
replaces on the GPU (through the C ABI)."""
import numpy as np
import pytest
import torch
from torch import nn

from oracle import nvfp4_ref as R

FLAGS = ("H3_KERNELS", "H3_NVFP4", "H3_FUSED_ROPE", "H3_FUSED_MODULATE", "H3_TL_ATTN",
         "H3_FUSED_SWIGLU", "H3_FUSED_GATE")


@pytest.fixture
def flags(monkeypatch):
    for f in FLAGS:
        monkeypatch.delenv(f, raising=False)

    def arm(*names):
        for n in names:
            monkeypatch.setenv(n, "1")
    return arm


def rel(a, b):
    a, b = a.detach().float(), b.detach().float()
    return float((a - b).abs().max() / b.abs().max())


# ------------------------------------------------------------------ CPU
def test_dispatch_surface(flags):
    from h3_engine_b200.kernels import _dispatch as D
    assert not D.MISS and repr(D.MISS) == "MISS"
    D.armed_counts(reset=True)
    assert D.enabled("H3_FUSED_ROPE") is False
    flags("H3_KERNELS")
    assert D.enabled("H3_FUSED_ROPE") and D.enabled("H3_NVFP4")
    assert D.armed_counts(reset=True) == {"H3_FUSED_ROPE": 1, "H3_NVFP4": 1}
    D.miss_counts(reset=True)
    # names with no kernel here, and arguments the kernels do not take (CPU tensors)
    assert D.try_call("gate_residual_gather", 1, 2, 3, 4) is D.MISS
    x = torch.zeros(1, 8, 2, 128, dtype=torch.bfloat16)
    cs = torch.zeros(8, 128)
    assert D.try_call("rope", x, cs, cs) is D.MISS
    assert D.miss_counts() == {"gate_residual_gather": 1, "rope": 1}


def test_flags_off_paths_are_the_stock_expressions(flags):
    """With no flag set (and on the CPU, where every call is MISS) the shims
    compute what the reference's stock code computes."""
    from h3_engine_b200.kernels import elementwise_norm_rope as ew
    from h3_engine_b200.kernels import ffn_qkvo_gemms as gm
    from h3_engine_b200.kernels import packed_self_attn as at
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, 16, 2, 64, generator=g)
    cos, sin = torch.randn(16, 32, generator=g), torch.randn(16, 32, generator=g)
    x1, x2 = x[..., :32].chunk(2, dim=-1)
    ref = torch.cat((x[..., :32] * cos[None, :, None] + torch.cat((-x2, x1), -1) * sin[None, :, None],
                     x[..., 32:]), -1)
    rope_ref = ref
    assert torch.allclose(ew.apply_rotary_emb(x, cos, sin), ref)
    norm = nn.RMSNorm(64, eps=1e-5)
    assert ew.norm_rope(norm, x, cos, sin) is None
    assert ew.norm_modulate(norm, x, cos, sin, torch.zeros(16, dtype=torch.long)) is None
    q = torch.randn(2, 8, 2, 64, generator=g)
    o = at.packed_self_attention(q, q, q)
    ref = torch.nn.functional.scaled_dot_product_attention(*(q.transpose(1, 2),) * 3).transpose(1, 2)
    assert torch.allclose(o, ref)
    lin = nn.Linear(64, 32, bias=False)
    y = torch.randn(4, 64, generator=g)
    assert torch.allclose(gm.out_projection(lin, y), lin(y))
    flags("H3_KERNELS")                       # armed, but CPU tensors are not covered
    assert torch.allclose(ew.apply_rotary_emb(x, cos, sin), rope_ref)
    assert torch.allclose(at.packed_self_attention(q, q, q), o)


def test_swiglu_weight_relayout_cpu():
    """The packed up-projection with rows in the SwiGLU epilogue's order:
    codes and block scales move with their rows, the global scale stays."""
    from h3_engine_b200 import nvfp4, ops
    from h3_engine_b200.kernels import ffn_qkvo_gemms as gm
    F, K = 128, 256
    g = torch.Generator().manual_seed(1)
    q = torch.randint(0, 256, (2 * F, K // 2), generator=g, dtype=torch.uint8)
    s_rows = torch.randint(0, 120, (2 * F, K // 16), generator=g, dtype=torch.uint8)
    w = nvfp4.NVFP4Weight.from_packed(q, nvfp4._swizzle(s_rows.view(torch.float8_e4m3fn)),
                                      2 * F, K, 0.5)

    class Lin:
        weight_nvfp4 = w
    lin = Lin()
    wq, wsf, wgs = gm._swiglu_weight(lin)
    perm = ops.swiglu_rows(F)
    assert torch.equal(wq, q[perm])
    assert torch.equal(nvfp4._unswizzle(wsf, 2 * F, K // 16), s_rows[perm])
    assert float(wgs) == 0.5
    assert gm._swiglu_weight(lin)[0] is wq          # cached on the module


# ------------------------------------------------------------------ GPU
def _tables(T, dims, dev):
    from h3_engine_b200.rope import rope_tables
    pos = torch.stack([torch.arange(T) % 7, torch.arange(T) % 5, torch.arange(T) % 3], 1)
    cos, sin = rope_tables(pos, dims)
    return cos.to(dev), sin.to(dev)


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,H,D,dims", [(1, 300, 4, 128, (44, 42, 42)),
                                          (2, 129, 3, 128, (16, 16, 16)),
                                          (1, 64, 2, 64, (8, 8, 16))])
def test_rope_shims_match_stock(cuda, flags, B, T, H, D, dims):
    from h3_engine_b200.kernels import _dispatch
    from h3_engine_b200.kernels import elementwise_norm_rope as ew
    g = torch.Generator().manual_seed(T)
    x = torch.randn(B, T, H, D, generator=g).to(torch.bfloat16).to(cuda)
    cos, sin = _tables(T, dims, cuda)
    norm = nn.RMSNorm(D, eps=1e-5).to(cuda).to(torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(D, generator=g))
    x0 = x.clone()
    ref_rope = ew.apply_rotary_emb(x, cos, sin)                  # flag off: stock
    ref_nr = ew._norm_rope_impl(x, norm.weight, 1e-5, cos, sin)
    flags("H3_FUSED_ROPE")
    _dispatch.miss_counts(reset=True)
    out_rope = ew.apply_rotary_emb(x, cos, sin)
    out_nr = ew.norm_rope(norm, x, cos, sin)
    assert _dispatch.try_call("norm_rope_h3", x, norm.weight, 1e-5, cos, sin) is not _dispatch.MISS
    assert _dispatch.miss_counts() == {}
    assert out_rope.shape == x.shape and out_nr.shape == x.shape
    assert rel(out_rope, ref_rope) <= 1e-2
    assert rel(out_nr, ref_nr) <= 1e-2
    assert torch.equal(x, x0)                                    # the input is not modified


@pytest.mark.gpu
def test_norm_modulate_shim_and_nvfp4_handoff(cuda, flags):
    from h3_engine_b200 import nvfp4, ops
    from h3_engine_b200.kernels import elementwise_norm_rope as ew
    g = torch.Generator().manual_seed(2)
    T, C = 333, 512
    x = torch.randn(1, T, C, generator=g).to(torch.bfloat16).to(cuda)
    scale = (0.1 * torch.randn(4, C, generator=g)).to(torch.bfloat16).to(cuda)
    shift = (0.1 * torch.randn(4, C, generator=g)).to(torch.bfloat16).to(cuda)
    idx = torch.randint(0, 4, (T,), generator=g).to(cuda)
    norm = nn.RMSNorm(C, eps=1e-6).to(cuda).to(torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(C, generator=g))
    assert ew.norm_modulate(norm, x, scale, shift, idx) is None      # flag off
    ref = ew._norm_modulate_impl(x, norm.weight, 1e-6, scale, shift, idx)
    flags("H3_FUSED_MODULATE")
    y = ew.norm_modulate(norm, x, scale, shift, idx)
    assert y.shape == x.shape and y.dtype == torch.bfloat16
    assert rel(y, ref) <= 1e-2
    # the NVFP4 form riding on y is exactly the quantization of y
    act = nvfp4.QuantizedActivation(y)
    q, sf, gs = ops.quantize(y.view(T, C), mpad=ops.pad_m(T))
    assert torch.equal(act.qdata.view(torch.uint8), q)
    assert torch.equal(act.scale_blocked.view(torch.uint8), sf)
    assert float(act.global_scale) == float(gs)
    assert act.qdata.data_ptr() == y._h3b_nvfp4[0].data_ptr()       # reused, not recomputed
    y.mul_(2)                                                       # written since: re-quantized
    act2 = nvfp4.QuantizedActivation(y)
    assert float(act2.global_scale) == 2 * float(gs)


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,H", [(1, 517, 2), (3, 200, 4)])
def test_attention_shim_matches_sdpa(cuda, flags, B, T, H):
    from h3_engine_b200.kernels import _dispatch
    from h3_engine_b200.kernels import packed_self_attn as at
    g = torch.Generator().manual_seed(B * T)
    q, k, v = (torch.randn(B, T, H, 128, generator=g).to(torch.bfloat16).to(cuda)
               for _ in range(3))
    ref = at.packed_self_attention(q, k, v)                          # flag off: SDPA
    flags("H3_TL_ATTN")
    out = at.packed_self_attention(q, k, v)
    assert out.shape == q.shape
    assert rel(out, ref) <= 1e-2
    flat = _dispatch.try_call("attention", q.reshape(B, T, -1), k.reshape(B, T, -1),
                              v.reshape(B, T, -1), H)
    assert torch.equal(flat.view(B, T, H, 128), out)
    mask = torch.ones(T, T, dtype=torch.bool, device=cuda)
    assert rel(at.packed_self_attention(q, k, v, mask), ref) <= 1e-2   # masked: SDPA path


class _SwiGLU(nn.Module):
    def __init__(self, d, f):
        super().__init__()
        self.proj = nn.Linear(d, 2 * f, bias=False)
        self.activation = nn.SiLU()

    def forward(self, x):
        h, gate = self.proj(x).chunk(2, dim=-1)
        return h * self.activation(gate)


class _FF(nn.Module):
    def __init__(self, d, f):
        super().__init__()
        self.net = nn.ModuleList([_SwiGLU(d, f), nn.Dropout(0.0), nn.Linear(f, d, bias=False)])

    def forward(self, x):
        for m in self.net:
            x = m(x)
        return x


@pytest.mark.gpu
def test_gemm_shims_on_quantized_linears(cuda, flags):
    from h3_engine_b200 import nvfp4
    from h3_engine_b200.kernels import ffn_qkvo_gemms as gm
    g = torch.Generator().manual_seed(3)
    T, d, f = 300, 512, 512
    x = torch.randn(1, T, d, generator=g).to(torch.bfloat16).to(cuda)

    def lin(n, k):
        m = nn.Linear(k, n, bias=False)
        with torch.no_grad():
            m.weight.copy_(0.05 * torch.randn(n, k, generator=g))
        return m.to(cuda).to(torch.bfloat16)
    to_q, to_k, to_v, to_out = lin(d, d), lin(d, d), lin(d, d), lin(d, d)
    ff = _FF(d, f).to(cuda).to(torch.bfloat16)
    with torch.no_grad():
        ff.net[0].proj.weight.copy_(0.05 * torch.randn(2 * f, d, generator=g))
        ff.net[2].weight.copy_(0.05 * torch.randn(d, f, generator=g))
    qq, qk, qv, qo = (nvfp4._QuantLinear(m) for m in (to_q, to_k, to_v, to_out))
    ff.net[0].proj = nvfp4._QuantLinear(ff.net[0].proj)
    ff.net[2] = nvfp4._QuantLinear(ff.net[2])
    # stock paths (flag off) already run the quantized linears one by one
    ref_qkv = (qq(x), qk(x), qv(x))
    ref_out = qo(x)
    ref_ff = ff(x)
    flags("H3_NVFP4")
    out_qkv = gm.qkv_projection(qq, qk, qv, x)
    for a, b in zip(out_qkv, ref_qkv):
        assert torch.equal(a, b)          # one shared activation quantization, same GEMM math
    assert torch.equal(gm.out_projection(qo, x), ref_out)
    y = gm.ffn(ff, x)
    assert y.shape == ref_ff.shape
    assert rel(y, ref_ff) <= 1e-2
    # against the oracle: the packed weights, activations quantized by the recipe
    def packed(w):
        return (w.qdata.cpu().numpy(),
                R.unswizzle(w.scale_u8.cpu().numpy(), w.out_features, w.in_features // 16),
                np.float32(float(w.global_scale)))
    qa, sa, ga = R.quantize(x.float().cpu().numpy()[0])
    u = R.bf16_round(R.gemm_ref(qa, sa, ga, *packed(ff.net[0].proj.weight_nvfp4), T, 2 * f)
                     .astype(np.float32))
    val, gate = u[:, :f], u[:, f:]
    h = R.bf16_round(val * R.bf16_round(gate / (1 + np.exp(-gate))))
    qh, sh, gh = R.quantize(h)
    yr = R.bf16_round(R.gemm_ref(qh, sh, gh, *packed(ff.net[2].weight_nvfp4), T, d)
                      .astype(np.float32))
    assert R.max_rel_err(y.float().cpu().numpy()[0], yr) <= 1e-2
