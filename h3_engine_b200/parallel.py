"""Multi-GPU layout of the DiT forward: CFG split, then token shards.

One process per GPU (torch.distributed over NCCL).  With N ranks:
  N = 1      both CFG branches on one GPU, stacked into one 2T-row pass;
  N = 2      one CFG branch per GPU, full sequence;
  N = 2P     one CFG branch per group of P GPUs, each holding T/P token rows.
Every GEMM, quantization and norm is row-independent, so token shards only
meet in attention: after qk-norm + RoPE each rank writes its K|V rows into its
chunk of a full-sequence buffer and one in-place all-gather over the token
group completes it (the only bulk exchange per block).  Every NVFP4
quantization first takes the max of its 4-byte amax over all ranks, so each
activation of the CFG batch keeps one global scale and every layout computes
the same bytes as the single-GPU run.  On NCCL runs that max goes through
peer memory (``PeerAmax``: one warp stores this rank's value into every
peer's slot array and polls its own, a bounded device-side wait, no host
collective); elsewhere (gloo) through an all-reduce.  The CFG combine exchanges each rank's
velocity rows with its peer in the other branch once per step.

``split_rows`` / ``ParallelLayout`` are pure host logic (tested on CPU with
gloo ranks); the collectives run on NCCL in GPU runs.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import torch_ops  # noqa: F401  (registers torch.ops.h3b)
from .blocks import SequenceShard


def split_rows(total: int, parts: int, index: int) -> tuple[int, int, int]:
    """Equal chunks of ``ceil(total/parts)`` rows: (row0, rows, chunk).  The
    last shard may be shorter (its chunk is padded in gathered buffers)."""
    chunk = -(-total // parts)
    row0 = min(index * chunk, total)
    rows = max(0, min(chunk, total - row0))
    return row0, rows, chunk


class PeerMemoryUnavailable(RuntimeError):
    """Peer memory could not be set up on some rank (no CUDA IPC / peer access)."""


class PeerAmax:
    """The max of a 4-byte fp32 amax over all ranks through peer memory.

    Each rank allocates a zeroed slot array of 2 * world 64-bit words
    (``h3b_peer_buffer_create``), the ranks swap its CUDA IPC handle once
    (``all_gather_object``) and map each other's (``h3b_peer_buffer_open``).
    Exchange number e (counted identically on every rank, because every rank
    quantizes the same activations in the same order) is one
    ``h3b_amax_exchange`` launch on the current stream: no NCCL kernel and no
    host synchronization per quantization.  A rank that never arrives makes
    the others' wait expire after ``limit_us`` with H3B_ERR_TIMEOUT recorded
    in the device error word (their amax stays local).  Every rank must call
    ``close`` (a collective) before the process group is destroyed."""

    def __init__(self, rank: int, world: int, device: torch.device, group=None,
                 limit_us: int = 30_000_000):
        """Collective over ``group``.  Raises ``PeerMemoryUnavailable`` on
        every rank, after undoing its own set-up, if any rank could not
        allocate, export or map a slot array."""
        import ctypes
        from . import _lib
        self.rank, self.world, self.limit_us, self.group = rank, world, limit_us, group
        lib = _lib.lib()
        handle = (ctypes.c_uint8 * 64)()
        own = ctypes.c_void_p()
        with torch.cuda.device(device):
            made = lib.h3b_peer_buffer_create(2 * world * 8, ctypes.byref(own), handle) == 0
        handles: list = [None] * world
        dist.all_gather_object(handles, bytes(handle) if made else None, group=group)
        ptrs, self._opened = [], []
        ok = all(h is not None for h in handles)
        with torch.cuda.device(device):
            for r in range(world):
                if not ok:
                    break
                if r == rank:
                    ptrs.append(own.value)
                    continue
                buf = (ctypes.c_uint8 * 64).from_buffer_copy(handles[r])
                p = ctypes.c_void_p()
                if lib.h3b_peer_buffer_open(buf, ctypes.byref(p)) != 0:
                    ok = False
                    break
                ptrs.append(p.value)
                self._opened.append(p.value)
        # every rank learns whether every rank is mapped
        flags: list = [None] * world
        dist.all_gather_object(flags, ok, group=group)
        self._own = own.value if made else None
        if not all(flags):
            self._release(lib)
            raise PeerMemoryUnavailable("a rank could not allocate, export or map its slot array")
        self.table = torch.tensor(ptrs, dtype=torch.int64, device=device)
        self.epoch = 0

    def _release(self, lib) -> None:
        import ctypes
        from . import _lib
        for p in self._opened:
            _lib.check(lib.h3b_peer_buffer_close(ctypes.c_void_p(p)), "h3b_peer_buffer_close")
        if self._own is not None:
            _lib.check(lib.h3b_peer_buffer_destroy(ctypes.c_void_p(self._own)),
                       "h3b_peer_buffer_destroy")
        self._own, self._opened = None, []

    def __call__(self, t: torch.Tensor) -> None:
        self.epoch += 1
        torch.ops.h3b.amax_exchange(t, self.table, self.rank, self.world, self.epoch,
                                    self.limit_us)

    def close(self) -> None:
        """Unmap the peers' arrays and free this rank's, after every rank's
        last exchange (a barrier over the group)."""
        from . import _lib
        if self._own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        self._release(_lib.lib())


@dataclass
class ParallelLayout:
    world: int
    rank: int
    cfg_parallel: int            # 1 or 2: CFG branches on separate GPUs
    token_parallel: int          # token shards per CFG branch
    branch: int                  # which CFG branch this rank computes (cfg_parallel == 2)
    token_rank: int
    token_group: object = None   # process group of this rank's token shards
    pair_group: object = None    # {this rank, its peer in the other branch}
    peer_amax: object = None     # PeerAmax over all ranks (NCCL runs)

    @staticmethod
    def plan(world: int, rank: int) -> "ParallelLayout":
        if world == 1:
            return ParallelLayout(1, 0, 1, 1, 0, 0)
        if world % 2:
            raise ValueError("multi-GPU runs split the CFG batch of 2: use an even GPU count")
        p = world // 2
        return ParallelLayout(world, rank, 2, p, rank // p, rank % p)

    def shard_rows(self, total: int) -> tuple[int, int, int]:
        return split_rows(total, self.token_parallel, self.token_rank)

    def build_groups(self) -> None:
        """Create the process groups (every rank must call this, same order)."""
        if self.world == 1:
            return
        p = self.token_parallel
        for b in range(2):
            ranks = list(range(b * p, (b + 1) * p))
            g = dist.new_group(ranks)
            if b == self.branch:
                self.token_group = g
        for t in range(p):
            ranks = [t, p + t]
            g = dist.new_group(ranks)
            if t == self.token_rank:
                self.pair_group = g
        # the amax max through peer memory on NCCL (GPU) runs;
        # H3B_AMAX_VIA=nccl keeps the NCCL all-reduce
        if dist.get_backend() == "nccl" and os.environ.get("H3B_AMAX_VIA", "peer") == "peer":
            dev = torch.device("cuda", torch.cuda.current_device())
            try:
                self.peer_amax = PeerAmax(self.rank, self.world, dev)
            except PeerMemoryUnavailable as e:
                # decided on every rank alike: the NCCL all-reduce instead
                import warnings
                warnings.warn(f"amax exchange through NCCL: {e}")
                self.peer_amax = None

    def close(self) -> None:
        """Release the peer-memory amax exchange (a collective: every rank,
        after its last step, before the process group is destroyed)."""
        if self.peer_amax is not None:
            self.peer_amax.close()
            self.peer_amax = None

    def sequence_shard(self, total: int) -> SequenceShard | None:
        """None on one GPU; otherwise this rank's shard with the K|V gather over
        its token group (absent without token sharding) and the amax max over
        all ranks (the CFG batch is one activation tensor)."""
        if self.world == 1:
            return None
        row0, rows, chunk = self.shard_rows(total)
        group = self.token_group

        def all_gather(full: torch.Tensor, local: torch.Tensor) -> None:
            # full: [>= chunk * P, C] buffer.  The send buffer is always this
            # rank's in-place slot token_rank * chunk (row0 equals it except
            # for trailing empty shards, where split_rows clamps row0 to the
            # total and a slice at row0 would overlap another rank's slot).
            dst = full[: chunk * self.token_parallel]
            slot = self.token_rank * chunk
            src = dst[slot: slot + chunk]
            dist.all_gather_into_tensor(dst, src, group=group)

        def reduce_max(t: torch.Tensor) -> None:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)

        if self.peer_amax is not None:
            reduce_max = self.peer_amax  # noqa: F811

        gather = all_gather if self.token_parallel > 1 else None
        return SequenceShard(row0, rows, total, gather, reduce_max, chunk=chunk,
                             parts=self.token_parallel)

    def exchange_velocity(self, v: torch.Tensor) -> torch.Tensor:
        """Returns the other CFG branch's velocity rows matching ``v``."""
        flat = v.contiguous().view(-1)
        out = torch.empty(2 * flat.numel(), dtype=v.dtype, device=v.device)
        dist.all_gather_into_tensor(out, flat, group=self.pair_group)
        return out.view((2,) + tuple(v.shape))[1 - self.branch]


def init_distributed(timeout_s: int = 300) -> tuple[int, int, int]:
    """(world, rank, local_rank) from the torchrun environment; joins NCCL."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        from datetime import timedelta
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", timeout=timedelta(seconds=timeout_s), device_id=dev)
    return world, rank, local
