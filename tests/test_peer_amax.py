"""The peer-memory amax exchange (h3b_amax_exchange) on one GPU.

The other ranks are stood in for by words written into this rank's slot
array beforehand (what a peer's store would leave there), so one kernel runs
alone and never waits on another launch.  Checked: the max over the posted
values, the epoch / half bookkeeping, and the bounded wait -- a slot that
nothing writes makes the wait expire, H3B_ERR_TIMEOUT reaches the host, the
amax stays local, and after that recorded failure later exchanges return
without waiting.  The exchange between real ranks is covered by the
multi-GPU layout test (tests/test_dit_model.py)."""
import struct
import time

import pytest
import torch

from h3_engine_b200 import _lib, torch_ops  # noqa: F401

pytestmark = pytest.mark.gpu


def _word(epoch: int, value: float) -> int:
    bits = struct.unpack("<I", struct.pack("<f", value))[0]
    w = (epoch << 32) | bits
    return w - (1 << 64) if w >= 1 << 63 else w       # as int64


def _setup(cuda, world):
    slots = torch.zeros(2 * world, dtype=torch.int64, device=cuda)
    # every rank's array is this one: this rank's stores land in it and the
    # "peers'" words are written by the test
    table = torch.full((world,), slots.data_ptr(), dtype=torch.int64, device=cuda)
    return slots, table


def test_exchange_takes_the_max_over_ranks(cuda):
    world, rank = 4, 1
    slots, table = _setup(cuda, world)
    for epoch, mine, peers in [(1, 1.5, [2.5, 0.25, 1.0]), (2, 3.0, [0.5, 2.0, 2.9]),
                               (3, 0.0, [0.0, 0.0, 7.0])]:
        half = (epoch & 1) * world
        others = [r for r in range(world) if r != rank]
        for r, v in zip(others, peers):
            slots[half + r] = _word(epoch, v)
        amax = torch.tensor([mine], dtype=torch.float32, device=cuda)
        torch.ops.h3b.amax_exchange(amax, table, rank, world, epoch, 1_000_000)
        torch.cuda.synchronize()
        assert _lib.device_error() == 0
        assert amax.item() == max([mine] + peers)
        assert slots[half + rank].item() == _word(epoch, mine)     # this rank's own store


def test_exchange_wait_is_bounded(cuda):
    world, rank = 2, 0
    slots, table = _setup(cuda, world)
    _lib.device_error()                                          # start clean
    slots[(1 & 1) * world + 1] = _word(1, 9.0)
    amax = torch.tensor([1.0], dtype=torch.float32, device=cuda)
    torch.ops.h3b.amax_exchange(amax, table, rank, world, 1, 1_000_000)
    assert _lib.device_error() == 0 and amax.item() == 9.0
    # exchange 3 uses the same half, where rank 1's word still carries epoch 1:
    # nothing arrives, the 20 ms bound expires
    amax.fill_(1.0)
    torch.ops.h3b.amax_exchange(amax, table, rank, world, 3, 20_000)
    torch.cuda.synchronize()
    assert amax.item() == 1.0                                    # left local
    # a recorded failure: the next exchange does not wait its 2 s bound
    t0 = time.perf_counter()
    torch.ops.h3b.amax_exchange(amax, table, rank, world, 5, 2_000_000)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 1.0
    assert _lib.device_error() == 5                              # H3B_ERR_TIMEOUT, cleared
    # the context stays usable: a completed exchange right after
    slots[(7 & 1) * world + 1] = _word(7, 4.0)
    torch.ops.h3b.amax_exchange(amax, table, rank, world, 7, 1_000_000)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0 and amax.item() == 4.0


def test_exchange_rejects_bad_arguments(cuda):
    slots, table = _setup(cuda, 2)
    amax = torch.zeros(1, dtype=torch.float32, device=cuda)
    for args in [(amax, table, 2, 2, 1, 1000), (amax, table, 0, 2, 0, 1000),
                 (amax, table, 0, 33, 1, 1000), (amax, table, 0, 2, 1, 0)]:
        with pytest.raises(RuntimeError):
            torch.ops.h3b.amax_exchange(*args)
