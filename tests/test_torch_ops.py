"""The torch custom-operator boundary (``torch.ops.h3b.*``).

CPU: every C-ABI compute entry point is registered as an operator with its
outputs declared mutated, CUDA-only (a CPU tensor is a dispatch error, not a
fallback), with a fake implementation, so tracing a caller in fake mode
records ``h3b`` nodes (what ``torch.compile`` / ``torch.export`` see).
GPU: a compiled NVFP4 linear (``fullgraph=True``, no graph break) gives the
eager bytes."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.fx.experimental.proxy_tensor import make_fx

from h3_engine_b200 import ops, torch_ops  # noqa: F401

OPS = {
    "amax_bf16": {"out"},
    "nvfp4_quantize": {"q", "sf", "gs_out"},
    "nvfp4_dequantize": {"out"},
    "nvfp4_gemm": {"out", "amax_out"},
    "rmsnorm_stats": {"rstd", "amax"},
    "rmsnorm_quantize": {"gs_out", "q", "sf", "y_out"},
    "qk_norm_rope": {"buf", "k_buf"},
    "attention_varlen": {"out"},
    "qk_norm_rope_out": {"q_out", "k_out"},
    "attention_qkv": {"out"},
    "gate_residual": {"out"},
    "ada_modulate": {"out"},
    "amax_exchange": {"amax"},
}


def test_every_entry_point_is_an_operator_with_declared_outputs():
    for name, outs in OPS.items():
        schema = getattr(torch.ops.h3b, name).default._schema
        mutated = {a.name for a in schema.arguments if a.alias_info is not None
                   and a.alias_info.is_write}
        assert mutated == outs, (name, mutated)
        assert len(schema.returns) == 0, name


def test_cpu_tensors_are_refused():
    x = torch.zeros(4, 64, dtype=torch.bfloat16)
    out = torch.zeros(1, dtype=torch.float32)
    with pytest.raises((NotImplementedError, RuntimeError)):
        torch.ops.h3b.amax_bf16(x, 4, 64, 64, out)
    with pytest.raises(ValueError):
        ops.amax(x)


def _linear(x, w):
    qa, sa, ga = ops.quantize(x, mpad=ops.pad_m(x.shape[0]))
    qb, sb, gb = ops.quantize(w, mpad=w.shape[0])
    return ops.gemm(qa, sa, ga, x.shape[0], qb, sb, gb, w.shape[0], x.shape[1])


def _norm_attention(x, gamma, qkv, cos, sin, wq, wk):
    q, sf, gs = ops.rmsnorm_quantize(x, gamma, 1e-6)
    ops.qk_norm_rope(qkv, 2, 128, q_off=0, k_off=256, wq=wq, wk=wk, eps=1e-6, cos=cos, sin=sin)
    o = ops.attention_varlen(qkv, 2, 128, [0, 100, 256], q_off=0, k_off=256, v_off=512)
    return q, sf, gs, o


def _targets(gm):
    return [str(n.target) for n in gm.graph.nodes if n.op == "call_function"]


def test_fake_tracing_records_h3b_nodes():
    with FakeTensorMode():
        x = torch.empty(300, 1024, dtype=torch.bfloat16, device="cuda")
        w = torch.empty(512, 1024, dtype=torch.bfloat16, device="cuda")
        y = _linear(x, w)
        assert y.shape == (300, 512) and y.dtype == torch.bfloat16
        xs = torch.empty(256, 512, dtype=torch.bfloat16, device="cuda")
        gamma = torch.empty(512, dtype=torch.bfloat16, device="cuda")
        qkv = torch.empty(256, 768, dtype=torch.bfloat16, device="cuda")
        cos = torch.empty(256, 128, dtype=torch.float32, device="cuda")
        sin = torch.empty(256, 128, dtype=torch.float32, device="cuda")
        wq = torch.empty(128, dtype=torch.bfloat16, device="cuda")
    t = _targets(make_fx(_linear, tracing_mode="fake")(x, w))
    assert t.count("h3b.nvfp4_quantize.default") == 2 and "h3b.nvfp4_gemm.default" in t
    t = _targets(make_fx(_norm_attention, tracing_mode="fake")(xs, gamma, qkv, cos, sin, wq, wq))
    for name in ("rmsnorm_stats", "rmsnorm_quantize", "qk_norm_rope", "attention_varlen"):
        assert f"h3b.{name}.default" in t, (name, t)


@pytest.mark.gpu
def test_compiled_linear_matches_eager(cuda):
    g = torch.Generator().manual_seed(9)
    x = torch.randn(300, 1024, generator=g).to(torch.bfloat16).to(cuda)
    w = (torch.randn(512, 1024, generator=g) * 0.02).to(torch.bfloat16).to(cuda)
    eager = _linear(x, w)
    compiled = torch.compile(_linear, fullgraph=True, backend="aot_eager")(x, w)
    torch.cuda.synchronize()
    assert torch.equal(eager, compiled)
