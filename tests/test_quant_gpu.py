"""GPU parity of the NVFP4 quantize / pack / unpack kernels against the CPU
oracle, through the C ABI.  Packed bytes, scales and unpacked bf16 must be
bit-exact."""
import numpy as np
import pytest
import torch

from h3_engine_b200 import ops
from oracle import nvfp4_ref as R
from tests.golden_util import load_golden

pytestmark = pytest.mark.gpu


def to_dev_bf16(x_f32: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x_f32, dtype=np.float32)).to(dev).to(torch.bfloat16)


def seeded_bf16(shape, seed, std=1.0, outlier_frac=0.0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g) * std
    if outlier_frac:
        idx = torch.randperm(x.numel(), generator=g)[: max(1, int(x.numel() * outlier_frac))]
        x.view(-1)[idx] *= 50.0
    return x.to(torch.bfloat16)


@pytest.mark.parametrize("case", ["randn", "ragged", "edge", "weight"])
@pytest.mark.parametrize("layout", [ops.SF_ROWMAJOR, ops.SF_SWIZZLED])
def test_quantize_matches_golden(cuda, case, layout):
    g = load_golden("nvfp4_golden.npz")
    x = to_dev_bf16(R.bf16_from_bits(g[f"{case}_x_bits"]), cuda)
    M, K = x.shape
    mpad = R.pad_m(M)
    q, sf, gs = ops.quantize(x, mpad=mpad, layout=layout)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), g[f"{case}_q"])
    want_sf = g[f"{case}_sf_swizzled"] if layout == ops.SF_SWIZZLED else g[f"{case}_sf"].reshape(-1)
    assert np.array_equal(sf.cpu().numpy(), want_sf)
    assert gs.cpu().numpy()[0] == g[f"{case}_gs"][0]
    deq = ops.dequantize(q, sf, gs, M, K, layout=layout, sf_rows=mpad)
    got = deq.float().cpu().numpy()
    assert np.array_equal(R.bf16_bits(got), g[f"{case}_deq_bits"])


@pytest.mark.parametrize("M,K", [(4096, 3072), (1000, 12288), (37, 64), (129, 320)])
def test_quantize_random_bitexact(cuda, M, K):
    x = seeded_bf16((M, K), seed=1, outlier_frac=0.001)
    xd = x.to(cuda)
    q, sf, gs = ops.quantize(xd, mpad=R.pad_m(M), layout=ops.SF_SWIZZLED)
    amax = ops.amax(xd)
    torch.cuda.synchronize()
    xf = x.float().numpy()
    assert amax.item() == float(np.abs(xf).max())
    rq, rsf, rgs = R.quantize(xf, mpad=R.pad_m(M))
    assert gs.item() == float(rgs)
    assert np.array_equal(q.cpu().numpy(), rq)
    assert np.array_equal(sf.cpu().numpy(), R.swizzle(rsf))


def test_quantize_strided_rows_and_forced_gs(cuda):
    base = seeded_bf16((200, 640), seed=9).to(cuda)
    view = base[:, 64:576]                    # ldx = 640 > K = 512
    q, sf, gs = ops.quantize(view, mpad=256, layout=ops.SF_ROWMAJOR, gs=1.0)
    torch.cuda.synchronize()
    rq, rsf, rgs = R.quantize(view.float().cpu().numpy(), mpad=256, gs=1.0)
    assert gs.item() == 1.0
    assert np.array_equal(q.cpu().numpy(), rq)
    assert np.array_equal(sf.cpu().numpy().reshape(256, -1), rsf)


def test_amax_and_empty_inputs(cuda):
    x = seeded_bf16((3, 64), seed=2).to(cuda)
    a = ops.amax(x)
    assert a.item() == x.float().abs().max().item()
    z = torch.zeros(0, 64, dtype=torch.bfloat16, device=cuda)
    assert ops.amax(z).item() == 0.0
    # M == 0 with padding: every row is padding -> zero codes, zero scales, gs = 1
    q, sf, gs = ops.quantize(z, mpad=128, layout=ops.SF_SWIZZLED)
    torch.cuda.synchronize()
    assert gs.item() == 1.0
    assert int(q.abs().sum()) == 0 and int(sf.sum()) == 0


def test_full_size_config1_properties(cuda):
    """Largest quant-microbench shape: [32768, 12288] with outliers.  The oracle
    checks a row sample bit-exactly (with the GPU's global scale, which must be
    max|x|/2688) and dequantize -> quantize is idempotent on the whole tensor."""
    M, K = 32768, 12288
    g = torch.Generator(device=cuda).manual_seed(1)
    x = torch.randn(M, K, device=cuda, generator=g, dtype=torch.float32)
    idx = torch.randint(0, M * K, (M * K // 1000,), device=cuda, generator=g)
    x.view(-1)[idx] *= 50.0
    x = x.to(torch.bfloat16)
    q, sf, gs = ops.quantize(x, mpad=M, layout=ops.SF_SWIZZLED)
    amax = x.float().abs().max()
    assert gs.item() == float(np.float32(amax.item()) / np.float32(2688.0))
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(0))[:48].sort().values
    xs = x[rows.to(cuda)].float().cpu().numpy()
    rq, rsf, _ = R.quantize(xs, gs=gs.item())
    assert np.array_equal(q[rows.to(cuda)].cpu().numpy(), rq)
    sf_rows = R.unswizzle(sf.cpu().numpy(), M, K // 16)[rows.numpy()]
    assert np.array_equal(sf_rows, rsf)
    deq = ops.dequantize(q, sf, gs, M, K, layout=ops.SF_SWIZZLED)
    q2, sf2, gs2 = ops.quantize(deq, mpad=M, layout=ops.SF_SWIZZLED, gs=gs.item())
    assert torch.equal(q2, q) and torch.equal(sf2, sf)
    del x, deq, q2
