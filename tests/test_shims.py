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
    # a name with no kernel, and arguments the kernels do not take (not
    # tensors, CPU tensors)
    assert D.try_call("no_such_row", 1) is D.MISS
    assert D.try_call("gate_residual_gather", 1, 2, 3, 4) is D.MISS
    x = torch.zeros(1, 8, 2, 128, dtype=torch.bfloat16)
    cs = torch.zeros(8, 128)
    assert D.try_call("rope", x, cs, cs) is D.MISS
    assert D.try_call("ada_modulate_gather", x, cs, cs, torch.zeros(8, dtype=torch.long)) is D.MISS
    assert D.miss_counts() == {"no_such_row": 1, "gate_residual_gather": 1, "rope": 1,
                               "ada_modulate_gather": 1}


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
    assert rel(at.packed_self_attention(q, k, v, mask), ref) <= 1e-2   # one document
    # key / value views of one projection output (row stride 3*H*D): read in place
    qkv = torch.cat([q.flatten(2), k.flatten(2), v.flatten(2)], dim=-1)
    qv, kv, vv = (qkv[..., i * H * 128:(i + 1) * H * 128].unflatten(-1, (H, 128)) for i in range(3))
    assert torch.equal(at.packed_self_attention(qv, kv, vv), out)


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,H", [(1, 400, 2), (2, 300, 3)])
def test_attention_shim_pad_mask_as_documents(cuda, flags, B, T, H):
    """The reference model's pad mask (is_pad[None, :] == is_pad[:, None],
    h3_inference/transformer/model.py:326-329) runs on the kernel as two
    documents of a permuted sequence; SDPA with the same mask is the bar."""
    from h3_engine_b200.kernels import _dispatch
    from h3_engine_b200.kernels import packed_self_attn as at
    g = torch.Generator().manual_seed(T + H)
    q, k, v = (torch.randn(B, T, H, 128, generator=g).to(torch.bfloat16).to(cuda)
               for _ in range(3))
    is_pad = torch.rand(T, generator=g) < 0.3
    mask = (is_pad[None, :] == is_pad[:, None]).to(cuda)
    causal = torch.tril(torch.ones(T, T, dtype=torch.bool, device=cuda))
    ref = at.packed_self_attention(q, k, v, mask)                    # flag off: SDPA
    ref_causal = at.packed_self_attention(q, k, v, causal)
    flags("H3_TL_ATTN")
    _dispatch.miss_counts(reset=True)
    out = at.packed_self_attention(q, k, v, mask)
    assert _dispatch.miss_counts() == {}
    assert rel(out, ref) <= 1e-2
    # a mask of another form stays on SDPA (counted as a miss)
    out2 = at.packed_self_attention(q, k, v, causal)
    assert _dispatch.miss_counts() == {"attention": 1}
    assert torch.equal(out2, ref_causal)


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,C,n", [(1, 300, 512, 3), (2, 129, 1024, 6)])
def test_gate_residual_and_ada_modulate_shims_bit_exact(cuda, flags, B, T, C, n):
    """The gathered gate + residual and modulation kernels give the stock
    bf16 expressions' bytes (torch rounds after every op; so do they)."""
    from h3_engine_b200.kernels import _dispatch
    from h3_engine_b200.kernels import elementwise_norm_rope as ew
    g = torch.Generator().manual_seed(C + n)
    x, y = (torch.randn(B, T, C, generator=g).to(torch.bfloat16).to(cuda) for _ in range(2))
    gate, scale, shift = ((0.3 * torch.randn(n, C, generator=g)).to(torch.bfloat16).to(cuda)
                          for _ in range(3))
    idx = torch.randint(0, n, (T,), generator=g).to(cuda)
    ref_g = ew.gate_residual(x, y, gate, idx)                        # flags off: stock
    ref_m = ew.ada_modulate(x, scale, shift, idx)
    flags("H3_FUSED_GATE", "H3_FUSED_MODULATE")
    _dispatch.miss_counts(reset=True)
    assert torch.equal(ew.gate_residual(x, y, gate, idx), ref_g)
    assert torch.equal(ew.ada_modulate(x, scale, shift, idx), ref_m)
    assert _dispatch.miss_counts() == {}
    assert torch.equal(_dispatch.try_call("gate_residual_gather", x, y, gate, idx), ref_g)
    assert torch.equal(_dispatch.try_call("ada_modulate_gather", x, scale, shift, idx), ref_m)


@pytest.mark.gpu
def test_rope_shim_is_out_of_place(cuda, flags):
    """norm_rope returns a new tensor and leaves its (strided) input as it was."""
    from h3_engine_b200.kernels import elementwise_norm_rope as ew
    g = torch.Generator().manual_seed(12)
    T, H = 257, 3
    qkv = torch.randn(1, T, 3 * H * 128, generator=g).to(torch.bfloat16).to(cuda)
    q = qkv[..., :H * 128].unflatten(-1, (H, 128))                  # a strided view
    norm = nn.RMSNorm(128, eps=1e-5).to(cuda).to(torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(128, generator=g))
    ang = torch.rand(T, 48, generator=g).to(cuda) * 6.28
    cos = torch.cat([ang.cos(), ang.cos()], 1)
    sin = torch.cat([ang.sin(), ang.sin()], 1)
    before = qkv.clone()
    ref = ew._norm_rope_impl(q, norm.weight, 1e-5, cos, sin)
    flags("H3_FUSED_ROPE")
    out = ew.norm_rope(norm, q, cos, sin)
    assert torch.equal(qkv, before)
    assert out.shape == q.shape and out.is_contiguous()
    assert rel(out, ref) <= 1e-2


@pytest.mark.gpu
def test_shims_take_reference_style_quantized_linears(cuda, flags):
    """Modules carrying the reference's own NVFP4 weight object (slots qdata_t
    and scale, no global scale: its two-level scheme) reach the kernels
    through shared_qkv / out_projection: global scale 1 on the GEMM."""
    from h3_engine_b200 import nvfp4, ops
    from h3_engine_b200.kernels import _dispatch
    from h3_engine_b200.kernels import ffn_qkvo_gemms as gm

    class _RefWeight:                         # the reference NVFP4Weight's slots
        __slots__ = ("qdata_t", "scale", "in_features", "out_features", "dtype")

    class _RefQuantLinear(nn.Module):         # the reference _QuantLinear's attributes
        def __init__(self, w):
            super().__init__()
            q, sf, _ = ops.quantize(w, mpad=w.shape[0], gs=1.0)
            rw = _RefWeight()
            rw.qdata_t = q.view(torch.float4_e2m1fn_x2).t()
            rw.scale = sf.view(torch.float8_e4m3fn)
            rw.out_features, rw.in_features = w.shape
            rw.dtype = torch.bfloat16
            self.weight_nvfp4 = rw
            self.in_features, self.out_features, self.calls = w.shape[1], w.shape[0], 0

    g = torch.Generator().manual_seed(13)
    T, d = 200, 512
    x = torch.randn(1, T, d, generator=g).to(torch.bfloat16).to(cuda)
    ws = [(0.05 * torch.randn(d, d, generator=g)).to(torch.bfloat16).to(cuda) for _ in range(4)]
    mods = [_RefQuantLinear(w) for w in ws]
    flags("H3_NVFP4")
    _dispatch.miss_counts(reset=True)
    q, k, v = gm.qkv_projection(mods[0], mods[1], mods[2], x)
    o = gm.out_projection(mods[3], x)
    assert _dispatch.miss_counts() == {}
    assert [m.calls for m in mods] == [1, 1, 1, 1]
    # the same GEMMs through this library's own weight objects at global scale 1
    for got, w in zip((q, k, v, o), ws):
        qw, sw, _ = ops.quantize(w, mpad=d, gs=1.0)
        mine = nvfp4.NVFP4Weight.from_packed(qw, sw, d, d, 1.0)
        assert torch.equal(got, nvfp4.QuantizedActivation(x).mm(mine))


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
