"""Property tests of the oracle's NVFP4 primitives (CPU, hypothesis): the
E2M1 rounding against an independent nearest-value search, the packing
round trip, the recipe's invariants, and agreement of the two CPU
restatements (numpy oracle, torch-CPU port) on random shapes and scales."""
import numpy as np
import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from oracle import cpu_torch as C
from oracle import nvfp4_ref as R

_MAGS = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
SETTINGS = settings(max_examples=60, deadline=None,
                    suppress_health_check=[HealthCheck.too_slow])


def _e2m1_by_search(v: float) -> int:
    """Nearest E2M1 magnitude, ties to the even code (low mantissa bit 0),
    saturating at 6, sign bit from the value."""
    a = min(abs(v), 6.0)
    d = np.abs(_MAGS - a)
    best = np.flatnonzero(d == d.min())
    code = int(best[0]) if len(best) == 1 else int(best[best % 2 == 0][0])
    return code | (8 if np.signbit(np.float32(v)) else 0)


@SETTINGS
@given(st.lists(st.floats(-20.0, 20.0, allow_nan=False, width=32), min_size=1, max_size=64))
def test_e2m1_is_nearest_ties_to_even(vals):
    v = np.array(vals, dtype=np.float32)
    got = R.e2m1_rne_satfinite(v)
    assert [int(c) for c in got] == [_e2m1_by_search(float(x)) for x in v]


@SETTINGS
@given(st.integers(1, 8), st.integers(1, 8), st.integers(0, 2**31 - 1))
def test_pack_unpack_round_trip(rows, halves, seed):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 16, size=(rows, 2 * halves), dtype=np.uint8)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    assert np.array_equal(R.unpack_codes(packed), codes)


@SETTINGS
@given(st.integers(1, 40), st.sampled_from([16, 64, 128, 256]),
       st.floats(1e-6, 1e4), st.integers(0, 2**31 - 1), st.booleans())
def test_recipe_invariants(rows, k, scale, seed, zero_rows):
    rng = np.random.default_rng(seed)
    x = R.bf16_round((rng.standard_normal((rows, k)) * scale).astype(np.float32))
    if zero_rows:
        x[::3] = 0.0
    q, sf, gs = R.quantize(x, mpad=R.pad_m(rows))
    assert q.shape == (R.pad_m(rows), k // 2) and sf.shape == (R.pad_m(rows), k // 16)
    amax = np.float32(np.abs(x).max())
    assert gs == (np.float32(amax / np.float32(2688.0)) if amax > 0 else np.float32(1.0))
    assert np.all(sf[:rows] <= 0x7E)                     # finite, non-negative e4m3
    assert not np.any(q[rows:]) and not np.any(sf[rows:])  # padding rows are zero
    deq = R.dequantize_f32(q, sf, gs)[:rows]
    xb, db = x.reshape(rows, -1, 16), deq.reshape(rows, -1, 16)
    bmax = np.abs(xb).max(-1, keepdims=True)
    assert np.all(np.abs(db - xb) <= 0.25 * bmax + 1e-30)
    assert np.all(db[bmax[..., 0] == 0] == 0)               # an all-zero block stays zero


@SETTINGS
@given(st.integers(1, 24), st.sampled_from([64, 128, 256]), st.floats(1e-3, 1e3),
       st.integers(0, 2**31 - 1))
def test_numpy_and_torch_restatements_agree(rows, k, scale, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, k)).astype(np.float32) * np.float32(scale)
    x.reshape(-1)[:: max(1, x.size // 7)] *= 50            # outliers
    x = R.bf16_round(x)
    q, sf, gs = R.quantize(x)
    codes, s, gs_t = C.quantize(torch.from_numpy(x))
    assert np.float32(gs_t) == gs
    assert np.array_equal(s.numpy(), sf)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).numpy()
    assert np.array_equal(packed, q)
