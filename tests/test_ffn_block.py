"""FFN sub-block: GPU (through the C ABI) vs the CPU oracle, plus the CPU
baseline port vs the oracle."""
import numpy as np
import pytest
import torch

from oracle import blocks_ref as B
from oracle import cpu_torch as C
from oracle import nvfp4_ref as R

TOL = 1e-2


def make(T, d, f, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, d, generator=g).to(torch.bfloat16)
    w1 = (torch.randn(f, d, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(d, f, generator=g) * 0.02).to(torch.bfloat16)
    b1 = (torch.randn(f, generator=g) * 0.01).to(torch.bfloat16)
    b2 = (torch.randn(d, generator=g) * 0.01).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    return x, w1, b1, w2, b2, gamma


def oracle_weights(w):
    q, s, g = R.quantize(w.float().numpy())
    return q, s, g


def test_cpu_port_matches_oracle_quantizer():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(64, 256, generator=g)
    x.view(-1)[::97] *= 50
    x = x.to(torch.bfloat16).float()
    codes, s, gs = C.quantize(x)
    q, sf, rgs = R.quantize(x.numpy())
    assert gs == float(rgs)
    assert np.array_equal(s.numpy(), sf)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).numpy()
    assert np.array_equal(packed, q)
    assert np.array_equal(C.dequantize(codes, s, gs).numpy(), R.dequantize_f32(q, sf, rgs))


def test_rmsnorm_oracle_matches_reference_golden():
    from tests.golden_util import load_golden
    g = load_golden("blocks_golden.npz")
    x = R.bf16_from_bits(g["rms_x_bits"])[0]
    w = R.bf16_from_bits(g["rms_gamma_bits"])
    y = B.rmsnorm(x, w, float(g["rms_eps"][0]))
    assert np.array_equal(R.bf16_bits(y), g["rms_y_bits"][0])


def test_cpu_port_ffn_matches_oracle():
    x, w1, b1, w2, b2, gamma = make(32, 256, 512, seed=3)
    blk = C.FFNBlockCPU(w1, b1, w2, b2, gamma, 1e-6)
    y = blk(x).float().numpy()
    ref, _, _ = B.ffn_block(x.float().numpy(), gamma.float().numpy(), 1e-6,
                            oracle_weights(w1), b1.float().numpy(), oracle_weights(w2),
                            b2.float().numpy())
    assert R.max_rel_err(y, ref) <= TOL


def test_cpu_port_swiglu_ffn_matches_oracle():
    """The timed CPU port of the reference-shape FFN half (SwiGLU) against the
    oracle's restatement (no modulation, gate or bias)."""
    g = torch.Generator().manual_seed(12)
    T, d, f = 48, 256, 256
    x = torch.randn(T, d, generator=g).to(torch.bfloat16)
    wu = (torch.randn(2 * f, d, generator=g) * 0.05).to(torch.bfloat16)
    wd = (torch.randn(d, f, generator=g) * 0.05).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    blk = C.FFNBlockCPU(wu, None, wd, None, gamma, 1e-5, act="swiglu")
    y = blk(x).float().numpy()
    ref, _ = B.swiglu_ffn_block_mod(x.float().numpy(), gamma.float().numpy(), 1e-5,
                                    oracle_weights(wu), oracle_weights(wd))
    assert R.max_rel_err(y, ref) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("T,d,f", [(256, 512, 2048), (200, 768, 1536)])
def test_ffn_block_matches_oracle(cuda, T, d, f):
    from h3_engine_b200.blocks import FFNBlock
    x, w1, b1, w2, b2, gamma = make(T, d, f, seed=2)
    blk = FFNBlock(w1.to(cuda), b1.to(cuda), w2.to(cuda), b2.to(cuda), gamma.to(cuda), 1e-6)
    y = blk(x.to(cuda)).float().cpu().numpy()
    ref, _, _ = B.ffn_block(x.float().numpy(), gamma.float().numpy(), 1e-6,
                            oracle_weights(w1), b1.float().numpy(), oracle_weights(w2),
                            b2.float().numpy())
    assert R.max_rel_err(y, ref) <= TOL


@pytest.mark.gpu
def test_rmsnorm_quantize_kernel(cuda):
    """Fused RMSNorm -> NVFP4: y within 1 bf16 ulp of the oracle norm, and the
    packed bytes bit-exact against the oracle quantizer applied to the GPU's y."""
    from h3_engine_b200 import ops
    g = torch.Generator().manual_seed(5)
    M, K = 300, 3072
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(K, generator=g)).to(torch.bfloat16)
    q, sf, gs, y = ops.rmsnorm_quantize(x.to(cuda), gamma.to(cuda), 1e-6, return_y=True)
    torch.cuda.synchronize()
    yg = y.float().cpu().numpy()
    yr = B.rmsnorm(x.float().numpy(), gamma.float().numpy(), 1e-6)
    ulp = np.abs(yr) * 2.0 ** -7
    assert np.all(np.abs(yg - yr) <= ulp + 1e-30)
    rq, rs, rgs = R.quantize(yg, mpad=q.shape[0])
    assert gs.item() == float(rgs)
    assert np.array_equal(q.cpu().numpy(), rq)
    assert np.array_equal(sf.cpu().numpy(), R.swizzle(rs))


@pytest.mark.gpu
def test_rmsnorm_modulated_and_long_rows(cuda):
    from h3_engine_b200 import ops
    g = torch.Generator().manual_seed(6)
    M, K = 129, 5376          # K > 3072 takes the re-read variant
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(K, generator=g)).to(torch.bfloat16)
    shift = (0.1 * torch.randn(6, K, generator=g)).to(torch.bfloat16)
    scale = (0.1 * torch.randn(6, K, generator=g)).to(torch.bfloat16)
    idx = torch.randint(0, 6, (M,), generator=g, dtype=torch.int32)
    q, sf, gs, y = ops.rmsnorm_quantize(x.to(cuda), gamma.to(cuda), 1e-5, shift=shift.to(cuda),
                                        scale=scale.to(cuda), mod_idx=idx.to(cuda), return_y=True)
    torch.cuda.synchronize()
    yr = B.rmsnorm(x.float().numpy(), gamma.float().numpy(), 1e-5, shift.float().numpy(),
                   scale.float().numpy(), idx.numpy())
    assert R.max_rel_err(y.float().cpu().numpy(), yr) <= 1e-2
    rq, rs, rgs = R.quantize(y.float().cpu().numpy(), mpad=q.shape[0])
    assert np.array_equal(q.cpu().numpy(), rq)
    assert np.array_equal(sf.cpu().numpy(), R.swizzle(rs))


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,ldx,n_mod", [
    (1, 256, 256, 2),          # one 256-column chunk, a single row
    (257, 2048, 2048, 5),      # ragged last CTA, random modulation rows
    (67, 3072, 3072, 0),       # the widest row held in registers by pass 1
    (1000, 4096, 4160, 3),     # pass 1 re-reads the row; strided rows
    (130, 4352, 4352, 0),
])
def test_rmsnorm_quantize_shapes(cuda, M, K, ldx, n_mod):
    """Both pass-1 variants, row strides and modulation tables: y within 1e-2
    of the oracle, the global scale = amax(y) / 2688 exactly, and the packed
    bytes bit-exact against the oracle quantizer applied to the GPU's y."""
    from h3_engine_b200 import ops
    g = torch.Generator().manual_seed(M + K)
    xw = torch.randn(M, ldx, generator=g).to(torch.bfloat16)
    x = xw[:, :K]
    gamma = (1 + 0.1 * torch.randn(K, generator=g)).to(torch.bfloat16)
    kw = {}
    mod = None
    if n_mod:
        shift = (0.1 * torch.randn(n_mod, K, generator=g)).to(torch.bfloat16)
        scale = (0.1 * torch.randn(n_mod, K, generator=g)).to(torch.bfloat16)
        idx = torch.randint(0, n_mod, (M,), generator=g, dtype=torch.int32)
        kw = dict(shift=shift.to(cuda), scale=scale.to(cuda), mod_idx=idx.to(cuda))
        mod = (shift.float().numpy(), scale.float().numpy(), idx.numpy())
    xd = xw.to(cuda)[:, :K]
    assert xd.stride(0) == ldx
    q, sf, gs, y = ops.rmsnorm_quantize(xd, gamma.to(cuda), 1e-6, return_y=True, **kw)
    torch.cuda.synchronize()
    yg = y.float().cpu().numpy()
    yr = B.rmsnorm(x.float().numpy(), gamma.float().numpy(), 1e-6, *(mod or ()))
    assert R.max_rel_err(yg, yr) <= 1e-2
    assert gs.item() == float(np.float32(np.abs(yg).max()) / np.float32(2688.0))
    rq, rs, rgs = R.quantize(yg, mpad=q.shape[0])
    assert gs.item() == float(rgs)
    assert np.array_equal(q.cpu().numpy(), rq)
    assert np.array_equal(sf.cpu().numpy(), R.swizzle(rs))


@pytest.mark.gpu
def test_ffn_block_full_size_row_sample(cuda):
    """The FFN sub-block at its configured size (32768 x 3072, FFN 12288): a
    row sample through the oracle, with the re-quantization global scale
    taken from the GPU (the oracle cannot run the full up-projection)."""
    from h3_engine_b200.blocks import FFNBlock
    T, d, f = 32768, 3072, 12288
    x, w1, b1, w2, b2, gamma = make(T, d, f, seed=2)
    blk = FFNBlock(w1.to(cuda), b1.to(cuda), w2.to(cuda), b2.to(cuda), gamma.to(cuda), 1e-6)
    xd = x.to(cuda)
    y = blk(xd)
    ws = blk._workspace(T, xd.device)
    gs_u = float(ws["gsu"].item())
    gs_h = float(ws["norm"]["gs"].item())
    torch.cuda.synchronize()
    # the global scales are the amaxes of the full tensors
    u = ws["u"]
    assert gs_u == float(np.float32(u.float().abs().max().item()) / np.float32(2688.0))
    rows = torch.randperm(T, generator=torch.Generator().manual_seed(1))[:64].sort().values
    xs = x[rows].float().numpy()
    h = B.rmsnorm(xs, gamma.float().numpy(), 1e-6)
    assert np.isclose(gs_h, float(np.float32(np.abs(B.rmsnorm(
        x.float().numpy(), gamma.float().numpy(), 1e-6)).max()) / np.float32(2688.0)), rtol=1e-2)
    u_r, _ = B.nvfp4_linear_from_bf16(h, *oracle_weights(w1), bias=b1.float().numpy(),
                                      act="gelu_tanh", gs_a=gs_h)
    y_r, _ = B.nvfp4_linear_from_bf16(u_r, *oracle_weights(w2), bias=b2.float().numpy(),
                                      residual=xs, gs_a=gs_u)
    assert R.max_rel_err(y[rows.to(cuda)].float().cpu().numpy(), y_r) <= TOL


@pytest.mark.gpu
@pytest.mark.parametrize("M,K", [(1000, 3072), (300, 5376), (129, 5888)])
def test_rmsnorm_modulated_cfg_halves(cuda, M, K):
    """Modulation rows in contiguous halves (the stacked CFG pair): CTAs whose
    rows share one modulation row use the shared-memory table path, the CTA
    at the boundary (and K beyond the table limit) the per-element path; y
    within 1e-2 of the oracle and the packed bytes bit-exact against the
    oracle quantizer applied to the GPU's y."""
    from h3_engine_b200 import ops
    g = torch.Generator().manual_seed(M + 7 * K)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(K, generator=g)).to(torch.bfloat16)
    shift = (0.1 * torch.randn(2, K, generator=g)).to(torch.bfloat16)
    scale = (0.1 * torch.randn(2, K, generator=g)).to(torch.bfloat16)
    idx = (torch.arange(M) >= M // 2 + 3).to(torch.int32)      # boundary inside a CTA
    q, sf, gs, y = ops.rmsnorm_quantize(x.to(cuda), gamma.to(cuda), 1e-6, shift=shift.to(cuda),
                                        scale=scale.to(cuda), mod_idx=idx.to(cuda), return_y=True)
    torch.cuda.synchronize()
    yg = y.float().cpu().numpy()
    yr = B.rmsnorm(x.float().numpy(), gamma.float().numpy(), 1e-6, shift.float().numpy(),
                   scale.float().numpy(), idx.numpy())
    assert R.max_rel_err(yg, yr) <= 1e-2
    assert gs.item() == float(np.float32(np.abs(yg).max()) / np.float32(2688.0))
    rq, rs, _ = R.quantize(yg, mpad=q.shape[0])
    assert np.array_equal(q.cpu().numpy(), rq)
    assert np.array_equal(sf.cpu().numpy(), R.swizzle(rs))
