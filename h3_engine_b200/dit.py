"""Random-init multimodal DiT forward on the sm_100a kernels.

The full-model configuration: 48 DiT blocks (attention half + GELU/bias FFN
half, hidden 3072, 24 heads x 128, FFN 12288, RMSNorm eps 1e-6), adaLN-zero
modulation per block (shift / scale / gate for each half: an NVFP4 linear
3072 -> 18432 of SiLU(temb), the block structure of
h3_inference/transformer/model.py:157-209 with the reference's
H3AdaLayerNormModulation at :40-49), a 256-d sinusoidal timestep embedding
(h3_inference/transformer/ops.py:8-33, flip_sin_to_cos, shift 0) through a
2-layer NVFP4 MLP, and a final adaLN-modulated RMSNorm + NVFP4 projection
giving the velocity.  The sequence is the packed [video | audio] token layout
(3D RoPE 44/42/42 over t/h/w, audio on 1-D positions, two attention
documents); tokens enter and leave in the hidden space (no patch embedding).

A denoising step evaluates the CFG pair (conditional: temb + a seeded
conditioning vector; unconditional: temb), combines
v = v_u + g (v_c - v_u) and takes the flow-matching Euler step
x <- x + (sigma_{i+1} - sigma_i) v on sigma = linspace(1, 0, steps + 1)
(the schedule of h3_inference/tests/equiv.py:50-79).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import ops
from .blocks import AttnBlock, DiTBlock, FFNBlock
from .nvfp4 import NVFP4Weight
from .parallel import ParallelLayout
from .rope import packed_positions, rope_tables


@dataclass
class DiTConfig:
    blocks: int = 48
    hidden: int = 3072
    heads: int = 24
    head_dim: int = 128
    ffn: int = 12288
    freq_dim: int = 256
    rope_dims: tuple[int, int, int] = (44, 42, 42)
    theta: float = 10000.0
    eps: float = 1e-6
    video_grid: tuple[int, int, int] = (21, 30, 52)
    audio_tokens: int = 1024
    guidance: float = 5.0

    @property
    def tokens(self) -> int:
        t, h, w = self.video_grid
        return t * h * w + self.audio_tokens

    def cu_seqlens(self) -> list[int]:
        v = self.video_grid[0] * self.video_grid[1] * self.video_grid[2]
        return [0, v, v + self.audio_tokens]

    def flops_per_eval(self) -> dict:
        """FLOPs of one model evaluation of one CFG branch."""
        T, d, f, hd = self.tokens, self.hidden, self.ffn, self.heads * self.head_dim
        cu = self.cu_seqlens()
        attn = sum(4 * hd * (b - a) ** 2 for a, b in zip(cu[:-1], cu[1:]))
        gemm = 2 * T * d * (3 * hd) + 2 * T * hd * d + 4 * T * d * f
        return {"nvfp4": self.blocks * gemm, "attention": self.blocks * attn}


def timestep_embedding(t: torch.Tensor, dim: int = 256, max_period: float = 10000.0):
    """Sinusoidal embedding, cos first (flip_sin_to_cos), frequency shift 0
    (h3_inference/transformer/ops.py:8-33 with the model's arguments)."""
    half = dim // 2
    exponent = -math.log(max_period) * torch.arange(half, dtype=torch.float32,
                                                    device=t.device) / half
    emb = t[:, None].float() * torch.exp(exponent)[None, :]
    return torch.cat([torch.cos(emb), torch.sin(emb)], dim=-1)


class _Linear:
    """NVFP4 linear on small row counts (timestep MLP, modulation tables)."""

    def __init__(self, w: torch.Tensor, b: torch.Tensor | None):
        self.w = NVFP4Weight(w)
        self.b = None if b is None else b.to(torch.bfloat16).contiguous()

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        x = x.to(torch.bfloat16).contiguous()
        q, sf, gs = ops.quantize(x, mpad=ops.pad_m(x.shape[0]))
        return ops.gemm(q, sf, gs, x.shape[0], self.w.qdata, self.w.scale_u8,
                        self.w.global_scale, self.w.out_features, self.w.in_features, bias=self.b)


class RandomDiT:
    """Seeded random-init weights (normal, std 0.02; norm weights 1 + N(0, 0.1);
    biases N(0, 0.01)), generated block by block on the GPU and quantized to
    NVFP4 immediately so only the packed weights stay resident."""

    def __init__(self, cfg: DiTConfig, device, seed: int = 4):
        self.cfg = cfg
        self.device = device
        g = torch.Generator(device=device).manual_seed(seed)
        d, f, HD = cfg.hidden, cfg.ffn, cfg.heads * cfg.head_dim

        def w(n, k, std=0.02):
            return (torch.randn(n, k, generator=g, device=device) * std).to(torch.bfloat16)

        def vec(n, mean=0.0, std=0.01):
            return (mean + std * torch.randn(n, generator=g, device=device)).to(torch.bfloat16)

        self.t1 = _Linear(w(d, cfg.freq_dim), vec(d))
        self.t2 = _Linear(w(d, d), vec(d))
        self.cond = vec(d, std=1.0)                 # conditioning of the CFG "cond" branch
        self.blocks: list[DiTBlock] = []
        self.ada: list[_Linear] = []
        self.workspace: dict = {}           # activation buffers shared by all blocks
        for _ in range(cfg.blocks):
            attn = AttnBlock(w(HD, d), w(HD, d), w(HD, d), w(d, HD), vec(d, 1.0, 0.1),
                             vec(cfg.head_dim, 1.0, 0.1), vec(cfg.head_dim, 1.0, 0.1), cfg.heads,
                             eps=cfg.eps, qk_eps=cfg.eps, workspace=self.workspace)
            ffn = FFNBlock(w(f, d), vec(f), w(d, f), vec(d), vec(d, 1.0, 0.1), eps=cfg.eps,
                           workspace=self.workspace)
            self.blocks.append(DiTBlock(attn, ffn))
            self.ada.append(_Linear(w(6 * d, d), vec(6 * d)))
        self.out_ada = _Linear(w(2 * d, d), vec(2 * d))
        self.out_gamma = vec(d, 1.0, 0.1)
        self.proj_out = _Linear(w(d, d), vec(d))
        self._rope = None
        self._sel: dict[tuple[int, ...], torch.Tensor] = {}   # CFG-branch selectors

    # ------------------------------------------------------------------ pieces
    def temb(self, timesteps: torch.Tensor) -> torch.Tensor:
        e = timestep_embedding(timesteps, self.cfg.freq_dim)
        return self.t2(torch.nn.functional.silu(self.t1(e).float()))

    def rope(self) -> tuple[torch.Tensor, torch.Tensor]:
        if self._rope is None:
            pos = packed_positions(self.cfg.video_grid, self.cfg.audio_tokens, self.device)
            self._rope = rope_tables(pos, self.cfg.rope_dims, self.cfg.theta)
        return self._rope

    def forward(self, x: torch.Tensor, temb_pair: torch.Tensor, rows: slice,
                branches: list[int], shard=None) -> torch.Tensor:
        """Velocity for the local rows ``x`` (the rows ``rows`` of each CFG
        branch in ``branches``, stacked).  ``temb_pair`` [2, d]: conditional and
        unconditional embeddings; the modulation tables are computed for the
        pair on every rank (one activation tensor, one global scale) and the
        local branches' rows selected."""
        cfg = self.cfg
        d = cfg.hidden
        T = cfg.tokens
        n = rows.stop - rows.start
        cos, sin = self.rope()
        cos, sin = cos[rows], sin[rows]
        nb = len(branches)
        if nb > 1:
            cos, sin = cos.repeat(nb, 1), sin.repeat(nb, 1)
            cu = []
            for b in range(nb):
                cu += [c + b * T for c in cfg.cu_seqlens()[(0 if b == 0 else 1):]]
            mod_idx = torch.arange(nb, device=x.device, dtype=torch.int32).repeat_interleave(n)
        else:
            cu = cfg.cu_seqlens()
            mod_idx = None
        key = tuple(branches)
        if key not in self._sel:          # cached: no host->device copy inside a step
            self._sel[key] = torch.tensor(branches, device=x.device)
        sel = self._sel[key]
        st = torch.nn.functional.silu(temb_pair.float())
        h = x
        buf = [torch.empty_like(x), torch.empty_like(x)]
        for i, (blk, ada) in enumerate(zip(self.blocks, self.ada)):
            m = ada(st).index_select(0, sel)               # [nb, 6d]
            mod = tuple(m[:, j * d:(j + 1) * d].contiguous() for j in range(6))
            h = blk(h, (cos, sin), cu, mod, mod_idx, out=buf[i & 1], shard=shard)
        mo = self.out_ada(st).index_select(0, sel)
        q, sf, gs = ops.rmsnorm_quantize(h, self.out_gamma, cfg.eps,
                                         shift=mo[:, :d].contiguous(),
                                         scale=mo[:, d:].contiguous(), mod_idx=mod_idx,
                                         amax_hook=None if shard is None else shard.reduce_max)
        w = self.proj_out.w
        return ops.gemm(q, sf, gs, h.shape[0], w.qdata, w.scale_u8, w.global_scale, d, d,
                        bias=self.proj_out.b)


class Sampler:
    """CFG flow-matching sampling of the packed sequence over a parallel layout."""

    def __init__(self, model: RandomDiT, layout: ParallelLayout, steps: int = 8):
        self.model = model
        self.layout = layout
        self.steps = steps
        self.sigmas = torch.linspace(1.0, 0.0, steps + 1)
        T = model.cfg.tokens
        row0, rows, _ = layout.shard_rows(T)
        self.rows = slice(row0, row0 + rows)
        self.shard = layout.sequence_shard(T)
        if layout.peer_amax is not None:
            # every rank has its model before the first device-side amax
            # exchange, whose wait for the other ranks is bounded
            torch.cuda.synchronize()
            dist.barrier()

    def step(self, x: torch.Tensor, i: int) -> torch.Tensor:
        """One denoising step on this rank's latent rows ``x`` [rows, d]."""
        t = torch.full((1,), float(self.sigmas[i]) * 1000.0, device=x.device)
        dt = float(self.sigmas[i + 1] - self.sigmas[i])
        return self.step_at(x, t, dt)

    def step_at(self, x: torch.Tensor, t: torch.Tensor, dt) -> torch.Tensor:
        """The step at timestep ``t`` (device [1]) with Euler increment ``dt``
        (a float or a device scalar, so a captured graph can be replayed for
        every step of the schedule)."""
        m, L = self.model, self.layout
        temb = m.temb(t).float()                           # [1, d]
        te = torch.cat([temb + m.cond.float(), temb]).to(torch.bfloat16)
        if L.cfg_parallel == 1:
            v2 = m.forward(torch.cat([x, x]), te, self.rows, [0, 1], self.shard)
            n = x.shape[0]
            v_c, v_u = v2[:n], v2[n:]
        else:
            v = m.forward(x, te, self.rows, [L.branch], self.shard)
            other = L.exchange_velocity(v)
            v_c, v_u = (v, other) if L.branch == 0 else (other, v)
        g = m.cfg.guidance
        v = v_u.float() + g * (v_c.float() - v_u.float())
        return (x.float() + dt * v).to(torch.bfloat16)

    def latent(self, seed: int = 4) -> torch.Tensor:
        """This rank's rows of the seeded initial latent (same on every layout)."""
        cfg = self.model.cfg
        g = torch.Generator(device=self.model.device).manual_seed(seed * 1000 + 7)
        x = torch.randn(cfg.tokens, cfg.hidden, generator=g, device=self.model.device)
        return x[self.rows].to(torch.bfloat16).contiguous()


class GraphedSampler:
    """``Sampler.step`` captured once into a CUDA graph and replayed for every
    step of the schedule (the one-evaluation graph of
    h3_inference/tests/kprofile.py:151-199).  Static input / output rows and
    device scalars for the timestep and the Euler increment are refreshed
    before each replay; the first call runs one eager step to warm every
    buffer and kernel attribute, then captures.  One GPU (a graph holding
    NCCL collectives is not built here)."""

    def __init__(self, sampler: Sampler):
        if sampler.layout.world != 1:
            raise ValueError("GraphedSampler captures the single-GPU layout")
        self.sampler = sampler
        self.graph: torch.cuda.CUDAGraph | None = None
        self.x_in = self.x_out = self.t = self.dt = None

    def _capture(self, x: torch.Tensor) -> None:
        s = self.sampler
        dev = x.device
        self.x_in = x.clone()
        self.t = torch.zeros(1, device=dev)
        self.dt = torch.zeros((), device=dev)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            s.step_at(self.x_in, self.t, self.dt)          # warm-up on the capture stream
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.x_out = s.step_at(self.x_in, self.t, self.dt)

    def step(self, x: torch.Tensor, i: int) -> torch.Tensor:
        s = self.sampler
        if self.graph is None:
            self._capture(x)
        self.x_in.copy_(x)
        self.t.fill_(float(s.sigmas[i]) * 1000.0)
        self.dt.fill_(float(s.sigmas[i + 1] - s.sigmas[i]))
        self.graph.replay()
        return self.x_out
