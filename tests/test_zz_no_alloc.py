"""The no-allocation RMSNorm -> NVFP4 entry point.

Callers such as inference servers that give every kernel a fixed, pre-planned
memory pool, or plugin hosts whose execute path must not call the allocator,
cannot hand the library the per-row scratch that the two-call form
(h3b_rmsnorm_stats + h3b_rmsnorm_quantize) needs.  h3b_rmsnorm_quantize_noalloc
keeps that scratch in a fixed array inside the library.  This file checks,
through the C ABI, that it produces the same bytes as the allocating entry
points on two calls in a row (the second call must not see the first call's
leftovers), and that it rejects row counts beyond its fixed limit.

Kept in its own file named to be collected last, so a failure here cannot stop
a run before the other tests have run.
"""
import ctypes

import pytest
import torch

from h3_engine_b200 import _lib, ops

NOALLOC_MAX_ROWS = 131072


def _noalloc(x, gamma, eps, *, shift=None, scale=None, idx=None):
    M, K = x.shape
    mpad = ops.pad_m(M)
    q = torch.full((mpad, K // 2), 0xAB, dtype=torch.uint8, device=x.device)
    sf = torch.full((mpad * (K // 16),), 0xCD, dtype=torch.uint8, device=x.device)
    gs = torch.zeros(1, dtype=torch.float32, device=x.device)
    p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    st = _lib.lib().h3b_rmsnorm_quantize_noalloc(
        p(x), M, K, x.stride(0), p(gamma), float(eps), p(shift), p(scale), p(idx), p(gs),
        p(q), p(sf), mpad, torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "h3b_rmsnorm_quantize_noalloc")
    return q, sf, gs


def test_noalloc_rejects_rows_beyond_its_fixed_scratch():
    lib = _lib.lib()
    dummy = ctypes.c_void_p(1 << 20)       # never dereferenced: the size check comes first
    st = lib.h3b_rmsnorm_quantize_noalloc(dummy, NOALLOC_MAX_ROWS + 1, 256, 256, dummy, 1e-6,
                                          None, None, None, None, dummy, dummy,
                                          NOALLOC_MAX_ROWS + 128, None)
    assert st == 1


@pytest.mark.gpu
def test_noalloc_matches_allocating_entry_points_twice(cuda):
    g = torch.Generator().manual_seed(21)
    # call 1: large values (large amax); call 2: small values with modulation,
    # a different row count and K -- stale scratch from call 1 would show.
    x1 = (torch.randn(1000, 3072, generator=g) * 40).to(torch.bfloat16).to(cuda)
    g1 = (1 + 0.1 * torch.randn(3072, generator=g)).to(torch.bfloat16).to(cuda)
    x2 = (torch.randn(300, 5376, generator=g) * 0.01).to(torch.bfloat16).to(cuda)
    g2 = (1 + 0.1 * torch.randn(5376, generator=g)).to(torch.bfloat16).to(cuda)
    sh = (0.1 * torch.randn(4, 5376, generator=g)).to(torch.bfloat16).to(cuda)
    sc = (0.1 * torch.randn(4, 5376, generator=g)).to(torch.bfloat16).to(cuda)
    idx = torch.randint(0, 4, (300,), generator=g, dtype=torch.int32).to(cuda)

    cases = [dict(x=x1, gamma=g1, eps=1e-6), dict(x=x2, gamma=g2, eps=1e-5, shift=sh, scale=sc,
                                                  idx=idx)]
    for c in cases:
        q, sf, gs = _noalloc(c["x"], c["gamma"], c["eps"], shift=c.get("shift"),
                             scale=c.get("scale"), idx=c.get("idx"))
        rq, rsf, rgs = ops.rmsnorm_quantize(c["x"], c["gamma"], c["eps"], shift=c.get("shift"),
                                            scale=c.get("scale"), mod_idx=c.get("idx"))
        torch.cuda.synchronize()
        assert gs.item() == rgs.item()
        assert torch.equal(q, rq)
        assert torch.equal(sf, rsf)


@pytest.mark.gpu
def test_noalloc_layout_edges(cuda):
    """The two edges of the fixed array: the largest legal row count (the amax
    slot right after the last per-row entry), compared bit for bit with the
    allocating entry points; and no rows at all with padding rows only (the
    padded codes and scales come out zero)."""
    g = torch.Generator().manual_seed(22)
    M, K = NOALLOC_MAX_ROWS, 256
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(cuda)
    gamma = (1 + 0.1 * torch.randn(K, generator=g)).to(torch.bfloat16).to(cuda)
    for _ in range(2):
        q, sf, gs = _noalloc(x, gamma, 1e-6)
        rq, rsf, rgs = ops.rmsnorm_quantize(x, gamma, 1e-6)
        torch.cuda.synchronize()
        assert gs.item() == rgs.item()
        assert torch.equal(q, rq)
        assert torch.equal(sf, rsf)
    del x, q, sf, rq, rsf

    K = 512
    g0 =torch.ones(K, dtype=torch.bfloat16, device=cuda)
    q = torch.full((128, K // 2), 0xAB, dtype=torch.uint8, device=cuda)
    sf = torch.full((128 * (K // 16),), 0xCD, dtype=torch.uint8, device=cuda)
    gs = torch.zeros(1, dtype=torch.float32, device=cuda)
    st = _lib.lib().h3b_rmsnorm_quantize_noalloc(
        None, 0, K, K, g0.data_ptr(), 1e-6, None, None, None, gs.data_ptr(), q.data_ptr(),
        sf.data_ptr(), 128, torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "h3b_rmsnorm_quantize_noalloc")
    torch.cuda.synchronize()
    assert int(q.count_nonzero()) == 0
    assert int(sf.count_nonzero()) == 0
