"""CPU tests of the oracle: pinned against torch's fp8 cast, the reference's
own CPU decode (committed golden fixtures) and restatements of the layouts."""
import numpy as np
import pytest
import torch

from oracle import nvfp4_ref as R
from tests.golden_util import load_golden


def test_e4m3_matches_torch_cast_everywhere():
    # every e4m3 value, every midpoint between neighbours, and random fp32
    grid = R.e4m3_to_f32(np.arange(0, 127, dtype=np.uint8)).astype(np.float64)
    mids = ((grid[:-1] + grid[1:]) / 2).astype(np.float32)
    rng = np.random.default_rng(0)
    rand = np.concatenate([rng.uniform(0, 470, 50000), np.exp2(rng.uniform(-14, 9, 50000))])
    v = np.concatenate([grid.astype(np.float32), mids, rand.astype(np.float32),
                        np.array([448.0, 460.0, 463.99, 464.0, 1e9], np.float32)])
    mine = R.e4m3_rne_satfinite(v)
    ref = torch.from_numpy(np.minimum(v, 448.0)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(mine, ref)
    assert np.array_equal(R.e4m3_rne_satfinite(grid.astype(np.float32)),
                          np.arange(0, 127, dtype=np.uint8))


def test_e2m1_ties_to_even_and_sign():
    v = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, 9.0,
                  0.2501, 0.7499, -0.1, -0.0, 0.0, -6.5], np.float32)
    want = [0, 2, 2, 4, 4, 6, 6, 7, 7, 1, 1, 8, 8, 0, 15]
    assert R.e2m1_rne_satfinite(v).tolist() == want
    # decoding every code through the reference LUT and re-encoding is the identity
    codes = np.arange(16, dtype=np.uint8)
    assert np.array_equal(R.e2m1_rne_satfinite(R.e2m1_decode(codes)), codes)


def test_reference_decode_pins_oracle_dequant():
    g = load_golden("nvfp4_golden.npz")
    assert np.array_equal(g["ref2_lut"], R.E2M1_LUT)
    deq = R.dequantize_f32(g["ref2_q"], g["ref2_sf"], np.float32(1.0))
    assert np.array_equal(deq, g["ref2_deq_f32"])


@pytest.mark.parametrize("case", ["randn", "ragged", "edge", "weight"])
def test_oracle_reproduces_golden(case):
    g = load_golden("nvfp4_golden.npz")
    x = R.bf16_from_bits(g[f"{case}_x_bits"])
    q, sf, gs = R.quantize(x, mpad=R.pad_m(x.shape[0]))
    assert np.array_equal(q, g[f"{case}_q"])
    assert np.array_equal(sf, g[f"{case}_sf"])
    assert np.float32(gs) == g[f"{case}_gs"][0]
    assert np.array_equal(R.swizzle(sf), g[f"{case}_sf_swizzled"])
    assert np.array_equal(R.bf16_bits(R.dequantize(q, sf, gs)[: x.shape[0]]), g[f"{case}_deq_bits"])


def _blocked_by_reshape(sf: np.ndarray) -> np.ndarray:
    """Second restatement of the 128x4 blocked layout via reshapes: pad, cut into
    (128 rows x 4 cols) tiles in row-major tile order, and inside a tile put row
    r = 32*i + j at [j][i]."""
    t = torch.from_numpy(sf)
    R_, C_ = t.shape
    rb, cb = -(-R_ // 128), -(-C_ // 4)
    p = torch.zeros(rb * 128, cb * 4, dtype=t.dtype)
    p[:R_, :C_] = t
    tiles = p.view(rb, 128, cb, 4).permute(0, 2, 1, 3)            # rb, cb, 128, 4
    tiles = tiles.reshape(rb, cb, 4, 32, 4).permute(0, 1, 3, 2, 4)  # rb, cb, 32(j), 4(i), 4
    return tiles.reshape(-1).numpy()


@pytest.mark.parametrize("shape", [(128, 4), (256, 8), (77, 12), (300, 20)])
def test_swizzle_two_restatements_agree(shape):
    rng = np.random.default_rng(1)
    sf = rng.integers(0, 255, size=shape, dtype=np.uint8)
    assert np.array_equal(R.swizzle(sf), _blocked_by_reshape(sf))
    assert np.array_equal(R.unswizzle(R.swizzle(sf), *shape), sf)


def test_quantize_error_bound_and_roundtrip():
    g = torch.Generator().manual_seed(3)
    x = R.bf16_round((torch.randn(64, 256, generator=g) * 3).numpy())
    q, sf, gs = R.quantize(x)
    deq = R.dequantize_f32(q, sf, gs)
    # every element is within half a code step of the block's scale grid,
    # plus the block-scale rounding (|bmax/s - 6| small): a loose bound of 1/4 of bmax
    xb = x.reshape(64, -1, 16)
    bmax = np.abs(xb).max(-1, keepdims=True)
    assert np.all(np.abs(deq.reshape(64, -1, 16) - xb) <= 0.25 * bmax + 1e-12)
    # re-quantizing the dequantized tensor with the same gs reproduces the codes
    q2, sf2, _ = R.quantize(deq, gs=gs)
    assert np.array_equal(sf2, sf)
    assert np.array_equal(q2, q)


def test_two_level_is_gs_one():
    g = torch.Generator().manual_seed(4)
    x = R.bf16_round(torch.randn(32, 128, generator=g).numpy())
    q, sf, gs = R.quantize(x, gs=1.0)
    assert gs == np.float32(1.0)
    s = R.e4m3_to_f32(sf)
    bmax = np.abs(x.reshape(32, -1, 16)).max(-1)
    assert np.array_equal(R.e4m3_rne_satfinite((bmax / np.float32(6.0)).astype(np.float32)), sf)
    assert np.all(s >= 0)


def test_linear_ref_close_to_bf16_linear():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(64, 256, generator=g)
    w = torch.randn(128, 256, generator=g) * 0.02
    y = R.linear_ref(x.numpy(), w.numpy())
    ref = (x @ w.T).numpy()
    cos = float(np.dot(y.ravel(), ref.ravel()) / np.linalg.norm(y) / np.linalg.norm(ref))
    assert cos > 0.98       # the reference's own self-check bar (h3_inference/nvfp4.py:170)
