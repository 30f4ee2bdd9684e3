"""Multi-GPU layout of the DiT forward: CFG split, then token shards.

One process per GPU (torch.distributed over NCCL).  With N ranks:
  N = 1      both CFG branches on one GPU, stacked into one 2T-row pass;
  N = 2      one CFG branch per GPU, full sequence;
  N = 2P     one CFG branch per group of P GPUs, each holding T/P token rows.
Every GEMM, quantization and norm is row-independent, so token shards only
meet in attention: after qk-norm + RoPE each rank writes its K|V rows into its
chunk of a full-sequence buffer and one in-place all-gather over the token
group completes it (the only bulk exchange per block).  Every NVFP4
quantization first max-all-reduces its 4-byte amax over all ranks, so each
activation of the CFG batch keeps one global scale and every layout computes
the same bytes as the single-GPU run.  The CFG combine exchanges each rank's
velocity rows with its peer in the other branch once per step.

``split_rows`` / ``ParallelLayout`` are pure host logic (tested on CPU with
gloo ranks); the collectives run on NCCL in GPU runs.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import torch
import torch.distributed as dist

from .blocks import SequenceShard


def split_rows(total: int, parts: int, index: int) -> tuple[int, int, int]:
    """Equal chunks of ``ceil(total/parts)`` rows: (row0, rows, chunk).  The
    last shard may be shorter (its chunk is padded in gathered buffers)."""
    chunk = -(-total // parts)
    row0 = min(index * chunk, total)
    rows = max(0, min(chunk, total - row0))
    return row0, rows, chunk


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
