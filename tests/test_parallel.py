"""Multi-GPU layout bookkeeping and collectives, on CPU gloo ranks."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from h3_engine_b200.parallel import ParallelLayout, split_rows


def test_split_rows_covers_sequence():
    for total in (1, 7, 33784, 67568):
        for parts in (1, 2, 3, 4, 8):
            got = [split_rows(total, parts, i) for i in range(parts)]
            chunk = got[0][2]
            assert all(c == chunk for _, _, c in got)
            covered = []
            for r0, n, _ in got:
                covered += list(range(r0, r0 + n)) if n else []
            assert covered == list(range(total))


def test_plan():
    assert ParallelLayout.plan(1, 0).cfg_parallel == 1
    for world in (2, 4, 8):
        for rank in range(world):
            L = ParallelLayout.plan(world, rank)
            assert L.cfg_parallel == 2 and L.token_parallel == world // 2
            assert L.branch == rank // (world // 2) and L.token_rank == rank % (world // 2)
    with pytest.raises(ValueError):
        ParallelLayout.plan(3, 0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, total, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        L = ParallelLayout.plan(world, rank)
        L.build_groups()
        sh = L.sequence_shard(total)
        # amax: max over every rank
        t = torch.tensor([float(rank + 1)])
        sh.reduce_max(t)
        assert t.item() == float(world)
        # K|V gather over the token group into the padded buffer
        if L.token_parallel > 1:
            assert sh.all_gather is not None
            C = 3
            full = torch.full((sh.buffer_rows(), C), -1.0)
            local = full[sh.row0:sh.row0 + sh.rows]
            local.copy_(torch.arange(sh.row0, sh.row0 + sh.rows).float()[:, None].repeat(1, C))
            sh.all_gather(full, local)
            assert torch.equal(full[:total, 0], torch.arange(total).float())
        else:
            assert sh.all_gather is None and sh.rows == total
        # CFG velocity exchange with the peer of the other branch
        v = torch.full((2, 2), float(L.branch * 10 + L.token_rank))
        other = L.exchange_velocity(v)
        assert other[0, 0].item() == float((1 - L.branch) * 10 + L.token_rank)
        q.put((rank, "ok"))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


# (8, 5): chunk 2 over 4 token shards, the last shard empty (its row0 is
# clamped to the total), so its in-place send slot is not at row0
@pytest.mark.parametrize("world,total", [(2, 37), (4, 37), (4, 40), (8, 37), (8, 33784), (8, 5)])
def test_collectives_on_gloo_ranks(world, total):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, total, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {r: "ok" for r in range(world)}
