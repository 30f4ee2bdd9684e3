"""Benchmark of the NVFP4 DiT hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl h3b|reference]
                    [--workload dit|ffn|attention|refblock|quant] [--attn-docs 32760,1024]

Default workload ("dit"): one denoising step of the full multimodal DiT --
48 blocks (hidden 3072, 24 heads x 128, FFN 12288 GELU/bias, adaLN-zero),
the packed sequence of 32760 video tokens (21 x 30 x 52 grid, 3D RoPE
44/42/42) + 1024 audio tokens (two attention documents), CFG batch of 2,
flow-matching Euler step; random-init weights (seed 4), synthetic latent.
On N GPUs: N = 1 both CFG branches stacked; N >= 2 CFG split and T/(N/2)
token shards per branch with one NCCL K|V all-gather per block (strong
scaling: the total work per step is fixed).

value       = whole-job TFLOP/s over every FLOP of the step (NVFP4 GEMMs +
              bf16 attention), step time = max over ranks of CUDA-event time;
ms_per_step = the denoising step; block_ms = ms_per_step / 48 (one DiT block
              of the CFG pair); nvfp4_gemm_tflops = GEMM flops / summed GEMM
              launch times (per GPU).
e2e         = the same metric through Sampler.step with the step's latent rows
              copied in from pinned host memory and the new latent copied back.

"ffn": the DiT FFN sub-block on 32768 tokens x 3072 (FFN 12288), one
independent shard per GPU (weak scaling, no collective).

"quant": the quantize/pack microbenchmark (amax + NVFP4 quantization of bf16
[M, K], M in {4096, 32768}, K in {3072, 12288}, 0.1 % outliers), GB/s against
the HBM roofline.

"refblock": one transformer block at the reference model's own shapes
(hidden 5376, 56 heads x 128, SwiGLU ffn 14336, 38247 tokens, one document),
one replica per GPU.

"attention": the packed varlen attention kernel alone (24 heads x 128, bf16,
documents of --attn-docs tokens, default the DiT packing 32760 + 1024) on a
seeded synthetic q|k|v activation, one replica per GPU; the kernel-level view
of the attention share of the DiT step and the small case profiled with ncu.

--impl reference: the reference's NVFP4 path cannot run on a CPU (its
quantizer is in the absent maiku package), so the timed CPU implementation is
the torch-CPU port of the recipe with the reference's own decode
(oracle/cpu_torch.py) on all host threads, on a bounded sample of query rows
(attention against full-length keys) extrapolated linearly to the workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "NVFP4 GEMM TFLOP/s/GPU & % FP4 peak; DiT block latency at 1/2/4/8 B200"
FFN_TOKENS, HIDDEN, FFN = 32768, 3072, 12288
# Per-launch DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of
# the kernel named in the roofline object, from one ncu capture each:
#   k_fmha: 639.9 MB read + 187.8 MB written = 827.6 MB for one launch on the
#     32760 + 1024-token packing (24 heads; q|k|v 622.7 MB read once, O
#     207.6 MB of which 187.8 MB reached DRAM inside the launch), i.e. per
#     token of the launch; the DiT launch (the CFG pair stacked, 2 x 33784
#     tokens) is the same per-token figure times its tokens.
#   k_gemm_nvfp4: FFN up 835.5 MB, down 639.4 MB at 32768 tokens (mean).
ATTN_TRAFFIC_PER_TOKEN = (639878656 + 187751424) / 33784
TRAFFIC_BYTES: dict[str, float | None] = {"k_fmha": ATTN_TRAFFIC_PER_TOKEN * 2 * 33784,
                                          "k_gemm_nvfp4": (835.5e6 + 639.4e6) / 2}


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"bf16_sustained": float(d["bf16_tflops_sustained"]), "bf16": float(d["bf16_tflops"]),
                "hbm": float(d["hbm_gbs"]), "source": "measured"}
    return {"bf16_sustained": 1400.0, "bf16": 1590.0, "hbm": 6650.0, "source": "fallback"}


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict:
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        load = [s for s in sm if smax and s > 0.3 * smax] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- workloads
class DiTWorkload:
    name = "dit"

    def __init__(self, dev, world: int, rank: int, steps_in_schedule: int = 8):
        from h3_engine_b200.dit import DiTConfig, RandomDiT, Sampler
        from h3_engine_b200.parallel import ParallelLayout

        self.cfg = DiTConfig()
        self.layout = ParallelLayout.plan(world, rank)
        self.layout.build_groups()
        self.model = RandomDiT(self.cfg, dev, seed=4)
        self.sampler = Sampler(self.model, self.layout, steps=steps_in_schedule)
        self.x = self.sampler.latent()
        self.i = 0
        f = self.cfg.flops_per_eval()
        self.step_flops = 2 * (f["nvfp4"] + f["attention"])     # CFG pair, whole job
        rows = self.sampler.rows.stop - self.sampler.rows.start
        branches = 2 if self.layout.cfg_parallel == 1 else 1
        T = self.cfg.tokens
        d, hd, ff = self.cfg.hidden, self.cfg.heads * self.cfg.head_dim, self.cfg.ffn
        # this rank's GEMM flops per step (block GEMMs of its rows)
        self.rank_gemm_flops = self.cfg.blocks * branches * rows * (
            2 * d * 3 * hd + 2 * hd * d + 4 * d * ff)
        cu = self.cfg.cu_seqlens()
        doc_of = [(a, b) for a, b in zip(cu[:-1], cu[1:])]
        r0, r1 = self.sampler.rows.start, self.sampler.rows.stop
        self.rank_attn_flops = self.cfg.blocks * branches * sum(
            4 * hd * max(0, min(b, r1) - max(a, r0)) * (b - a) for a, b in doc_of)
        self.attn_launches_per_step = self.cfg.blocks
        # DRAM bytes of one attention launch on this rank, from the full-size
        # capture (ATTN_TRAFFIC_PER_TOKEN): per query row its q read (6144 B)
        # and 5557 B of its output written inside the launch; per key row
        # 12797 B read (K|V once, +4 % re-reads)
        q_rows, kv_rows = rows * branches, T * branches
        self.attn_traffic = q_rows * (6144 + 187751424 / 33784) + kv_rows * (
            (639878656 - 6144 * 33784) / 33784)
        # the block GEMM shapes of the stacked CFG pair (rows padded to 128 by the GEMM)
        M2 = 2 * T
        self.library_shapes = {"qkv": (M2, 3 * hd, d), "out": (M2, d, hd), "up": (M2, ff, d),
                               "down": (M2, d, ff), "square_8192": (8192, 8192, 8192)}
        self.config = self.describe(world)
        # CUDA events around this rank's collectives (the K|V gather on its
        # side stream, the amax max on the main stream), recorded only while
        # the timers are set (the timed steps)
        self._comm, self.comm_last = None, None
        sh = self.sampler.shard
        if sh is not None:
            def timed(kind, fn):
                def run(*a):
                    ev = self._comm
                    if ev is None:
                        return fn(*a)
                    st = torch.cuda.current_stream()
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record(st)
                    fn(*a)
                    e1.record(st)
                    ev.setdefault(kind, []).append((e0, e1))
                return run
            if sh.all_gather is not None:
                sh.all_gather = timed("kv_gather", sh.all_gather)
            sh.reduce_max = timed("amax_max", sh.reduce_max)

    def comm_summary(self, steps: int) -> dict | None:
        """Per timed step on this rank: calls and stream time of each
        collective (a collective's time includes waiting for the other
        ranks)."""
        if not self.comm_last:
            return None
        out = {}
        for kind, evs in self.comm_last.items():
            tot = sum(a.elapsed_time(b) for a, b in evs)
            out[kind] = {"calls_per_step": len(evs) / steps, "ms_per_step": tot / steps,
                         "us_per_call": tot / max(len(evs), 1) * 1e3}
        return out

    @staticmethod
    def describe(world: int) -> dict:
        from h3_engine_b200.dit import DiTConfig
        from h3_engine_b200.parallel import ParallelLayout
        cfg, L = DiTConfig(), ParallelLayout.plan(world, 0)
        return {"workload": "multimodal DiT denoising step (CFG pair): 48 blocks x (attention "
                            "sub-block + GELU FFN sub-block), adaLN-zero, seed 4",
                "tokens": cfg.tokens, "documents": cfg.cu_seqlens(), "hidden": cfg.hidden,
                "heads": cfg.heads, "head_dim": cfg.head_dim, "ffn": cfg.ffn, "cfg_batch": 2,
                "parallelism": f"cfg{L.cfg_parallel} x tokens{L.token_parallel}",
                "l2": "working set several GB per step > 126 MB L2 (no flush needed)"}

    def set_timers(self, gemm, attn):
        for b in self.model.blocks:
            b.attn.gemm_events, b.ffn.gemm_events = gemm, gemm
            b.attn.attn_events = attn
        if gemm is not None:
            self._comm = {}
        else:
            self.comm_last, self._comm = self._comm, None

    def step(self):
        self.x = self.sampler.step(self.x, self.i % self.sampler.steps)
        self.i += 1

    def e2e_setup(self):
        self.x_h = self.x.cpu().pin_memory()
        self.y_h = torch.empty_like(self.x_h).pin_memory()
        self.x_d = torch.empty_like(self.x)
        return self.x_h.numel() * 2, self.y_h.numel() * 2

    def e2e_step(self):
        self.x_d.copy_(self.x_h, non_blocking=True)
        y = self.sampler.step(self.x_d, self.i % self.sampler.steps)
        self.i += 1
        self.y_h.copy_(y, non_blocking=True)


class FFNWorkload:
    name = "ffn"

    def __init__(self, dev, world: int, rank: int, tokens: int = FFN_TOKENS):
        from h3_engine_b200.blocks import FFNBlock
        g = torch.Generator(device="cpu").manual_seed(2)
        w1 = (torch.randn(FFN, HIDDEN, generator=g) * 0.02).to(torch.bfloat16).to(dev)
        w2 = (torch.randn(HIDDEN, FFN, generator=g) * 0.02).to(torch.bfloat16).to(dev)
        b1 = (torch.randn(FFN, generator=g) * 0.01).to(torch.bfloat16).to(dev)
        b2 = (torch.randn(HIDDEN, generator=g) * 0.01).to(torch.bfloat16).to(dev)
        gamma = (1 + 0.1 * torch.randn(HIDDEN, generator=g)).to(torch.bfloat16).to(dev)
        self.blk = FFNBlock(w1, b1, w2, b2, gamma, 1e-6)
        gd = torch.Generator(device=dev).manual_seed(2000 + rank)
        self.x = torch.randn(tokens, HIDDEN, generator=gd, device=dev).to(torch.bfloat16)
        self.y = torch.empty_like(self.x)
        self.step_flops = world * 4.0 * tokens * HIDDEN * FFN
        self.rank_gemm_flops = 4.0 * tokens * HIDDEN * FFN
        self.rank_attn_flops = 0
        self.config = self.describe(world, tokens)

    @staticmethod
    def describe(world: int, tokens: int = FFN_TOKENS) -> dict:
        return {"workload": "DiT FFN sub-block (seed 2): RMSNorm -> NVFP4 GEMM up 3072->12288 "
                            "(+bias, GELU-tanh) -> NVFP4 re-quant -> NVFP4 GEMM down (+bias) "
                            "-> residual", "tokens_per_gpu": tokens, "hidden": HIDDEN,
                "ffn": FFN, "parallelism": f"token-sharded x{world}, weights replicated",
                "l2": "working set ~1.3 GB per step > 126 MB L2 (no flush needed)"}

    def set_timers(self, gemm, attn):
        self.blk.gemm_events = gemm

    def step(self):
        self.blk(self.x, out=self.y)

    def e2e_setup(self):
        self.x_h = self.x.cpu().pin_memory()
        self.y_h = torch.empty_like(self.x_h).pin_memory()
        self.x_d = torch.empty_like(self.x)
        return self.x_h.numel() * 2, self.y_h.numel() * 2

    def e2e_step(self):
        self.x_d.copy_(self.x_h, non_blocking=True)
        self.blk(self.x_d, out=self.y)
        self.y_h.copy_(self.y, non_blocking=True)


class AttentionWorkload:
    name = "attention"
    HEADS, HEAD_DIM = 24, 128

    def __init__(self, dev, world: int, rank: int, docs: list[int]):
        H, D = self.HEADS, self.HEAD_DIM
        T = sum(docs)
        self.cu = [0]
        for n in docs:
            self.cu.append(self.cu[-1] + n)
        g = torch.Generator(device=dev).manual_seed(3000 + rank)
        self.qkv = torch.randn(T, 3 * H * D, generator=g, device=dev).to(torch.bfloat16)
        self.out = torch.empty(T, H * D, device=dev, dtype=torch.bfloat16)
        fl = sum(4 * H * D * n * n for n in docs)
        self.step_flops = world * fl
        self.rank_gemm_flops = 0
        self.rank_attn_flops = fl
        self.events = None
        self.config = self.describe(world, docs)

    @classmethod
    def describe(cls, world: int, docs: list[int]) -> dict:
        cu = [0]
        for n in docs:
            cu.append(cu[-1] + n)
        qkv_mb = cu[-1] * 3 * cls.HEADS * cls.HEAD_DIM * 2 / 1e6
        return {"workload": "packed varlen attention (bf16 q|k|v activation, 24 heads x 128, "
                            "one softmax(QK^T / sqrt(d)) V per document)",
                "documents": cu, "heads": cls.HEADS, "head_dim": cls.HEAD_DIM,
                "parallelism": f"replicas x{world}",
                "l2": f"q|k|v {qkv_mb:.0f} MB per launch"}

    def set_timers(self, gemm, attn):
        self.events = attn

    def _run(self, qkv):
        from h3_engine_b200 import ops
        H, D = self.HEADS, self.HEAD_DIM
        if self.events is not None:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
        ops.attention_varlen(qkv, H, D, self.cu, q_off=0, k_off=H * D, v_off=2 * H * D,
                             out=self.out)
        if self.events is not None:
            b.record()
            self.events.append((a, b))

    def step(self):
        self._run(self.qkv)

    def e2e_setup(self):
        self.x_h = self.qkv.cpu().pin_memory()
        self.y_h = torch.empty_like(self.out, device="cpu").pin_memory()
        self.x_d = torch.empty_like(self.qkv)
        return self.x_h.numel() * 2, self.y_h.numel() * 2

    def e2e_step(self):
        self.x_d.copy_(self.x_h, non_blocking=True)
        self._run(self.x_d)
        self.y_h.copy_(self.out, non_blocking=True)


class RefBlockWorkload:
    """One transformer block at the reference model's own shapes
    (h3_inference/transformer/model.py:211-230: hidden 5376, 56 heads x 128,
    SwiGLU ffn 14336, eps 1e-5, 16/16/16 RoPE, three modality tables) on the
    38247-token sequence of its production cell, one document, random-init
    weights (seed 5)."""
    name = "refblock"
    C, H, D, F, TOKENS = 5376, 56, 128, 14336, 38247

    def __init__(self, dev, world: int, rank: int):
        from h3_engine_b200.blocks import AttnBlock, DiTBlock, FFNBlock
        from h3_engine_b200.rope import reference_dims, rope_tables
        C, H, D, F, T = self.C, self.H, self.D, self.F, self.TOKENS
        HD = H * D
        g = torch.Generator(device=dev).manual_seed(5 + 1000 * rank)

        def w(n, k):
            return (torch.randn(n, k, generator=g, device=dev) / k ** 0.5).to(torch.bfloat16)

        def vec(n, mean, std):
            return (mean + std * torch.randn(n, generator=g, device=dev)).to(torch.bfloat16)

        self.ws: dict = {}
        attn = AttnBlock(w(HD, C), w(HD, C), w(HD, C), w(C, HD), vec(C, 1.0, 0.1),
                         vec(D, 1.0, 0.1), vec(D, 1.0, 0.1), heads=H, eps=1e-5, qk_eps=1e-5,
                         workspace=self.ws)
        ffn = FFNBlock(w(2 * F, C), None, w(C, F), None, vec(C, 1.0, 0.1), eps=1e-5,
                       workspace=self.ws, act="swiglu")
        self.blk = DiTBlock(attn, ffn)
        self.mod = tuple(((0.5 if j in (2, 5) else 0.0)
                          + 0.1 * torch.randn(3, C, generator=g, device=dev)).to(torch.bfloat16)
                         for j in range(6))
        n_vid = T - 2048
        self.idx = torch.cat([torch.zeros(n_vid), torch.ones(1024), 2 * torch.ones(1024)]).to(
            torch.int32).to(dev)
        pos = torch.stack([torch.arange(T) // 1024, (torch.arange(T) // 32) % 32,
                           torch.arange(T) % 32], dim=1).float().to(dev)
        self.rope = rope_tables(pos, reference_dims(16), 10000.0)
        self.x = torch.randn(T, C, generator=g, device=dev).to(torch.bfloat16)
        self.y = torch.empty_like(self.x)
        self.rank_gemm_flops = self.gemm_flops()
        self.rank_attn_flops = 4 * HD * T * T
        self.step_flops = world * (self.rank_gemm_flops + self.rank_attn_flops)
        self.attn_traffic = T * (3 * HD * 2 + HD * 2)    # q|k|v read once, O written
        self.config = self.describe(world)

    @classmethod
    def gemm_flops(cls) -> int:
        C, HD, F, T = cls.C, cls.H * cls.D, cls.F, cls.TOKENS
        return 2 * T * C * 3 * HD + 2 * T * HD * C + 2 * T * C * 2 * F + 2 * T * F * C

    @classmethod
    def flops(cls) -> int:
        """NVFP4 GEMM + attention flops of one block."""
        return cls.gemm_flops() + 4 * cls.H * cls.D * cls.TOKENS * cls.TOKENS

    @classmethod
    def describe(cls, world: int) -> dict:
        return {"workload": "one H3TransformerBlock at the reference model's shapes: RMSNorm + "
                            "gather-modulate, NVFP4 QKV (56 x 128 heads), qk-norm + 16/16/16 RoPE, "
                            "attention over the whole sequence, gated residual, SwiGLU FFN 14336",
                "tokens": cls.TOKENS, "hidden": cls.C, "heads": cls.H, "head_dim": cls.D,
                "ffn": cls.F, "parallelism": f"replicas x{world}",
                "l2": "working set several GB per step > 126 MB L2 (no flush needed)"}

    def set_timers(self, gemm, attn):
        self.blk.attn.gemm_events = self.blk.ffn.gemm_events = gemm
        self.blk.attn.attn_events = attn

    def step(self):
        self.blk(self.x, self.rope, [0, self.TOKENS], self.mod, self.idx, out=self.y)

    def e2e_setup(self):
        self.x_h = self.x.cpu().pin_memory()
        self.y_h = torch.empty_like(self.x_h).pin_memory()
        self.x_d = torch.empty_like(self.x)
        return self.x_h.numel() * 2, self.y_h.numel() * 2

    def e2e_step(self):
        self.x_d.copy_(self.x_h, non_blocking=True)
        self.blk(self.x_d, self.rope, [0, self.TOKENS], self.mod, self.idx, out=self.y)
        self.y_h.copy_(self.y, non_blocking=True)


class RefShimsWorkload:
    """The same reference-shape block, built as a module tree with the
    reference's module names (norm1, attn.{to_q,to_k,to_v,norm_q,norm_k,
    to_out.0}, norm2, ff.net.{0.proj,2}), its six linears swapped by
    ``nvfp4.quantize_blocks``, and run through the row shims of
    ``h3_engine_b200.kernels`` in the order H3TransformerBlock.forward calls
    them (h3_inference/transformer/model.py:81-106,176-209) with H3_KERNELS=1:
    the reference-API (drop-in) path, every row on a kernel."""
    name = "refblock-shims"
    C, H, D, F, TOKENS = RefBlockWorkload.C, RefBlockWorkload.H, RefBlockWorkload.D, \
        RefBlockWorkload.F, RefBlockWorkload.TOKENS

    def __init__(self, dev, world: int, rank: int):
        from torch import nn

        from h3_engine_b200 import nvfp4
        from h3_engine_b200.rope import reference_dims, rope_tables
        os.environ["H3_KERNELS"] = "1"
        C, H, D, F, T = self.C, self.H, self.D, self.F, self.TOKENS
        HD = H * D
        g = torch.Generator(device=dev).manual_seed(5 + 1000 * rank)

        def lin(n, k):
            m = nn.Linear(k, n, bias=False, device=dev, dtype=torch.bfloat16)
            with torch.no_grad():
                m.weight.copy_(torch.randn(n, k, generator=g, device=dev) / k ** 0.5)
            return m

        def rms(n):
            m = nn.RMSNorm(n, eps=1e-5, device=dev, dtype=torch.bfloat16)
            with torch.no_grad():
                m.weight.copy_(1 + 0.1 * torch.randn(n, generator=g, device=dev))
            return m

        blk = nn.Module()
        blk.norm1, blk.norm2 = rms(C), rms(C)
        blk.attn = nn.Module()
        blk.attn.heads = H
        blk.attn.to_q, blk.attn.to_k, blk.attn.to_v = lin(HD, C), lin(HD, C), lin(HD, C)
        blk.attn.norm_q, blk.attn.norm_k = rms(D), rms(D)
        blk.attn.to_out = nn.ModuleList([lin(C, HD), nn.Dropout(0.0)])
        up = nn.Module()
        up.proj, up.activation = lin(2 * F, C), nn.SiLU()
        blk.ff = nn.Module()
        blk.ff.net = nn.ModuleList([up, nn.Dropout(0.0), lin(C, F)])
        model = nn.Module()
        model.transformer_blocks = nn.ModuleList([blk])
        nvfp4.quantize_blocks(model, self_check=False)
        self.blk = blk
        self.tables = tuple(((0.5 if j in (2, 5) else 0.0)
                             + 0.1 * torch.randn(3, C, generator=g, device=dev)).to(torch.bfloat16)
                            for j in range(6))
        n_vid = T - 2048
        self.idx = torch.cat([torch.zeros(n_vid), torch.ones(1024), 2 * torch.ones(1024)]).to(
            torch.long).to(dev)
        pos = torch.stack([torch.arange(T) // 1024, (torch.arange(T) // 32) % 32,
                           torch.arange(T) % 32], dim=1).float().to(dev)
        self.rope = rope_tables(pos, reference_dims(16), 10000.0)
        self.x = torch.randn(1, T, C, generator=g, device=dev).to(torch.bfloat16)
        self.rank_gemm_flops = RefBlockWorkload.gemm_flops()
        self.rank_attn_flops = 4 * HD * T * T
        self.step_flops = world * (self.rank_gemm_flops + self.rank_attn_flops)
        self.attn_traffic = T * (3 * HD * 2 + HD * 2)
        self.attn_events = None
        self.config = self.describe(world)

    @classmethod
    def describe(cls, world: int) -> dict:
        d = RefBlockWorkload.describe(world)
        d["workload"] = ("one H3TransformerBlock at the reference model's shapes through the "
                         "reference-API row shims (norm_modulate, qkv_projection, norm_rope, "
                         "packed_self_attention, out_projection, gate_residual, ffn) with "
                         "H3_KERNELS=1")
        return d

    def set_timers(self, gemm, attn):
        self.attn_events = attn

    def _forward(self, x):
        from h3_engine_b200 import ops
        from h3_engine_b200.kernels import elementwise_norm_rope as ew
        from h3_engine_b200.kernels import ffn_qkvo_gemms as gm
        from h3_engine_b200.kernels import packed_self_attn as at
        blk, idx, cos_sin = self.blk, self.idx, self.rope
        shift_a, scale_a, gate_a, shift_m, scale_m, gate_m = self.tables
        h = ew.norm_modulate(blk.norm1, x, scale_a, shift_a, idx)
        a = blk.attn
        q, k, v = gm.qkv_projection(a.to_q, a.to_k, a.to_v, h)
        q, k, v = (t.unflatten(-1, (a.heads, -1)) for t in (q, k, v))
        q = ew.norm_rope(a.norm_q, q, *cos_sin)
        k = ew.norm_rope(a.norm_k, k, *cos_sin)
        ev = self.attn_events
        if ev is not None:
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record()
        o = at.packed_self_attention(q, k, v, None)
        if ev is not None:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record()
            ev.append((e0, e1))
        o = gm.out_projection(a.to_out[0], o.flatten(2, 3).type_as(q))
        x = ew.gate_residual(x, o, gate_a, idx)
        h = ew.norm_modulate(blk.norm2, x, scale_m, shift_m, idx)
        return ew.gate_residual(x, gm.ffn(blk.ff, h), gate_m, idx)

    def step(self):
        from h3_engine_b200.kernels import _dispatch
        _dispatch.miss_counts(reset=True)
        self.y = self._forward(self.x)
        if _dispatch.miss_counts():
            raise RuntimeError(f"a row shim fell back to torch: {_dispatch.miss_counts()}")

    def e2e_setup(self):
        self.x_h = self.x.cpu().pin_memory()
        self.y_h = torch.empty_like(self.x_h).pin_memory()
        self.x_d = torch.empty_like(self.x)
        return self.x_h.numel() * 2, self.y_h.numel() * 2

    def e2e_step(self):
        self.x_d.copy_(self.x_h, non_blocking=True)
        y = self._forward(self.x_d)
        self.y_h.copy_(y, non_blocking=True)


class QuantWorkload:
    """The quantize / pack microbenchmark: amax + NVFP4 quantization (codes,
    blocked e4m3 scales, fp32 global scale) of bf16 [M, K] for M in {4096,
    32768} and K in {3072, 12288}, values N(0, 1) with 0.1 % of entries x50
    (seed 1).  Algorithmic bytes 4.5625 per element: the amax read (2 B), the
    quantization read (2 B), codes (0.5 B) and scales (0.0625 B)."""
    name = "quant"
    SHAPES = ((4096, 3072), (4096, 12288), (32768, 3072), (32768, 12288))

    def __init__(self, dev, world: int, rank: int):
        from h3_engine_b200 import ops
        self.ops = ops
        g = torch.Generator(device=dev).manual_seed(1 + 1000 * rank)
        self.xs, self.outs = [], []
        for M, K in self.SHAPES:
            x = torch.randn(M, K, generator=g, device=dev)
            hot = torch.rand(M, K, generator=g, device=dev) < 1e-3
            x = torch.where(hot, x * 50, x).to(torch.bfloat16)
            self.xs.append(x)
            self.outs.append((torch.empty(M, K // 2, dtype=torch.uint8, device=dev),
                              torch.empty(M * K // 16, dtype=torch.uint8, device=dev),
                              torch.zeros(1, device=dev), torch.empty(1, device=dev)))
        elems = sum(M * K for M, K in self.SHAPES)
        self.bytes_per_step = 4.5625 * elems
        self.quant_bytes = 2.5625 * elems            # the quantization kernel alone
        self.step_bytes = world * self.bytes_per_step
        self.rank_gemm_flops = self.rank_attn_flops = 0
        self.events = None
        self.config = self.describe(world)

    @classmethod
    def describe(cls, world: int) -> dict:
        return {"workload": "NVFP4 quantize/pack (amax + codes + blocked e4m3 scales + fp32 "
                            "global scale), N(0,1) with 0.1% outliers x50, seed 1",
                "shapes": [list(s) for s in cls.SHAPES], "parallelism": f"replicas x{world}",
                "l2": "1.1 GB of inputs per step > 126 MB L2 (no flush needed)"}

    def set_timers(self, gemm, attn):
        self.events = attn

    def _run(self, xs):
        ops = self.ops
        for x, (q, sf, amax, gs) in zip(xs, self.outs):
            amax.zero_()
            ops.amax(x, out=amax)
            if self.events is not None:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
            ops.quantize(x, mpad=x.shape[0], amax_t=amax, q_out=q, sf_out=sf, gs_out=gs)
            if self.events is not None:
                b.record()
                self.events.append((a, b))

    def step(self):
        self._run(self.xs)

    def unpack_rate(self, pk, reps: int = 10) -> dict:
        """The unpack of config 1 (codes + block scales + global scale ->
        bf16, 2.5625 B per element), CUDA events over ``reps`` passes of the
        four shapes after the timed region."""
        ops = self.ops
        outs = [torch.empty_like(x) for x in self.xs]

        def run():
            for x, (q, sf, _, gs), o in zip(self.xs, self.outs, outs):
                ops.dequantize(q, sf, gs, x.shape[0], x.shape[1], out=o)
        run()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            run()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / reps
        gbs = 2.5625 * sum(x.numel() for x in self.xs) / (ms * 1e-3) / 1e9
        return {"kernel": "h3b::k_nvfp4_dequantize<swizzled>", "ms_per_pass": ms,
                "achieved": gbs, "unit": "GB/s", "frac": gbs / pk["hbm"]}

    def roofline(self, pk, steps, ms, kernel_ms):
        achieved = self.quant_bytes * steps / (kernel_ms * 1e-3) / 1e9
        return {"bound": "hbm", "kernel": "h3b::k_nvfp4_quantize<swizzled>", "achieved": achieved,
                "peak": pk["hbm"], "unit": "GB/s", "frac": achieved / pk["hbm"],
                "peak_source": f"hbm_gbs of {pk['source']} MEASURED_PEAKS.json",
                "traffic": None, "algorithmic_bytes_per_step": self.quant_bytes,
                "whole_step_gbs": self.bytes_per_step / (ms * 1e-3) / 1e9,
                "whole_step_frac": self.bytes_per_step / (ms * 1e-3) / 1e9 / pk["hbm"]}

    def e2e_setup(self):
        self.x_h = [x.cpu().pin_memory() for x in self.xs]
        self.x_d = [torch.empty_like(x) for x in self.xs]
        self.q_h = [torch.empty_like(o[0], device="cpu").pin_memory() for o in self.outs]
        return (sum(x.numel() * 2 for x in self.xs),
                sum(o[0].numel() + o[1].numel() + 4 for o in self.outs))

    def e2e_step(self):
        for xh, xd in zip(self.x_h, self.x_d):
            xd.copy_(xh, non_blocking=True)
        self._run(self.x_d)
        for qh, o in zip(self.q_h, self.outs):
            qh.copy_(o[0], non_blocking=True)


# ----------------------------------------------------------------------------- CPU
CPU_SAMPLE_SECONDS = 10.0


def _timed_repeat(fn, min_seconds: float) -> tuple[float, int]:
    """Seconds per call of ``fn`` averaged over as many calls as fill
    ``min_seconds`` (at least one), after one untimed call."""
    fn()
    n, t0 = 0, time.perf_counter()
    while True:
        fn()
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            return el / n, n


def cpu_dit_estimate(sample_rows: int, min_seconds: float = CPU_SAMPLE_SECONDS) -> dict:
    """Extrapolated CPU time of the DiT step from a sample of query rows: the
    attention half (rows x all keys) and the FFN half of one block on
    ``sample_rows`` rows, repeated for ``min_seconds`` of CPU work, scaled to
    2 x T rows x 48 blocks."""
    from h3_engine_b200.dit import DiTConfig
    from oracle.cpu_torch import AttnRowsCPU, FFNBlockCPU

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = DiTConfig()
    T = cfg.tokens
    attn = AttnRowsCPU(cfg.hidden, cfg.heads, cfg.head_dim, T)
    g = torch.Generator().manual_seed(4)
    w = lambda n, k: (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)  # noqa: E731
    ffn = FFNBlockCPU(w(cfg.ffn, cfg.hidden), torch.zeros(cfg.ffn), w(cfg.hidden, cfg.ffn),
                      torch.zeros(cfg.hidden), torch.ones(cfg.hidden), cfg.eps)
    x = torch.randn(sample_rows, cfg.hidden, generator=g).to(torch.bfloat16)
    pos = torch.randint(0, 50, (sample_rows, 3), generator=g).float()
    from h3_engine_b200.rope import rope_tables
    cos, sin = rope_tables(pos, cfg.rope_dims, cfg.theta)
    dt, n = _timed_repeat(lambda: ffn(attn(x, cos, sin)), min_seconds)
    step_s = dt * (2 * T / sample_rows) * cfg.blocks
    f = cfg.flops_per_eval()
    flops = 2 * (f["nvfp4"] + f["attention"])
    return {"value": flops / step_s / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "port", "s_per_step": step_s,
            "sample": (f"{sample_rows} query rows of one block (attention against all {T} keys "
                       f"+ FFN) x {n} repeats, {dt * n:.1f} s of CPU work, "
                       f"{dt:.2f} s per sample, extrapolated linearly to 2 x {T} rows x "
                       f"{cfg.blocks} blocks")}


def cpu_ffn_run(sample_tokens: int, min_seconds: float = CPU_SAMPLE_SECONDS) -> dict:
    from oracle.cpu_torch import FFNBlockCPU

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator(device="cpu").manual_seed(2)
    w1 = (torch.randn(FFN, HIDDEN, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(HIDDEN, FFN, generator=g) * 0.02).to(torch.bfloat16)
    blk = FFNBlockCPU(w1, torch.zeros(FFN), w2, torch.zeros(HIDDEN), torch.ones(HIDDEN), 1e-6)
    x = torch.randn(sample_tokens, HIDDEN, generator=g).to(torch.bfloat16)
    dt, n = _timed_repeat(lambda: blk(x), min_seconds)
    return {"value": 4.0 * sample_tokens * HIDDEN * FFN / dt / 1e12, "unit": "TFLOP/s",
            "cores": torch.get_num_threads(), "kind": "port", "s_per_step": dt * FFN_TOKENS / sample_tokens,
            "sample": (f"{sample_tokens} of {FFN_TOKENS} tokens x {n} repeats, "
                       f"{dt * n:.1f} s of CPU work")}


def cpu_quant_run(sample_rows: int, min_seconds: float = CPU_SAMPLE_SECONDS) -> dict:
    """The quantize microbenchmark on the CPU port: amax + NVFP4 quantization
    of ``sample_rows`` rows of each of its four shapes (same value
    distribution), repeated for ``min_seconds``; GB/s of the 4.5625 algorithmic
    bytes per element, the unit of the GPU line."""
    from oracle.cpu_torch import quantize

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(1)
    xs = []
    for _, K in QuantWorkload.SHAPES:
        x = torch.randn(sample_rows, K, generator=g)
        hot = torch.rand(sample_rows, K, generator=g) < 1e-3
        xs.append(torch.where(hot, x * 50, x).to(torch.bfloat16))

    def run():
        for x in xs:
            quantize(x)                   # amax of the sample, then codes and scales

    dt, n = _timed_repeat(run, min_seconds)
    sample_elems = sum(x.numel() for x in xs)
    full_elems = sum(M * K for M, K in QuantWorkload.SHAPES)
    return {"value": 4.5625 * sample_elems / dt / 1e9, "unit": "GB/s",
            "cores": torch.get_num_threads(), "kind": "port",
            "s_per_step": dt * full_elems / sample_elems,
            "sample": (f"{sample_rows} rows of each of the 4 shapes x {n} repeats, "
                       f"{dt * n:.1f} s of CPU work")}


def cpu_attention_run(docs: list[int], sample_rows: int,
                      min_seconds: float = CPU_SAMPLE_SECONDS) -> dict:
    """Packed attention on the CPU: softmax(Q K^T / sqrt(d)) V in fp32 torch
    ops for ``sample_rows`` query rows of each document against all of that
    document's keys (24 heads x 128), repeated for ``min_seconds``; TFLOP/s of
    4 * H * D * rows * keys, scaled to every query row for ms_per_step."""
    H, D = AttentionWorkload.HEADS, AttentionWorkload.HEAD_DIM
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(3)
    parts = []
    for n in docs:
        rows = min(sample_rows, n)
        q = torch.randn(H, rows, D, generator=g).to(torch.bfloat16).float()
        k = torch.randn(H, n, D, generator=g).to(torch.bfloat16).float()
        v = torch.randn(H, n, D, generator=g).to(torch.bfloat16).float()
        parts.append((q, k, v))

    def run():
        for q, k, v in parts:
            p = torch.softmax(q @ k.transpose(1, 2) * D ** -0.5, dim=-1)
            (p @ v).to(torch.bfloat16)

    dt, n_rep = _timed_repeat(run, min_seconds)
    sample_flops = sum(4 * H * D * q.shape[1] * k.shape[1] for q, k, _ in parts)
    full_flops = sum(4 * H * D * n * n for n in docs)
    return {"value": sample_flops / dt / 1e12, "unit": "TFLOP/s",
            "cores": torch.get_num_threads(), "kind": "port",
            "s_per_step": dt * full_flops / sample_flops,
            "sample": (f"{sample_rows} query rows per document x all its keys, {n_rep} repeats, "
                       f"{dt * n_rep:.1f} s of CPU work")}


def cpu_refblock_run(sample_rows: int, min_seconds: float = CPU_SAMPLE_SECONDS) -> dict:
    """The reference-shape block on the CPU port: attention half (sample rows
    against all 38247 keys, 56 x 128 heads) and SwiGLU FFN half on
    ``sample_rows`` rows, repeated for ``min_seconds``, scaled to every row."""
    from h3_engine_b200.rope import reference_dims, rope_tables
    from oracle.cpu_torch import AttnRowsCPU, FFNBlockCPU

    W = RefBlockWorkload
    torch.set_num_threads(os.cpu_count() or 1)
    attn = AttnRowsCPU(W.C, W.H, W.D, W.TOKENS, seed=5)
    g = torch.Generator().manual_seed(5)
    w = lambda n, k: (torch.randn(n, k, generator=g) / k ** 0.5).to(torch.bfloat16)  # noqa: E731
    ffn = FFNBlockCPU(w(2 * W.F, W.C), None, w(W.C, W.F), None, torch.ones(W.C), 1e-5,
                      act="swiglu")
    x = torch.randn(sample_rows, W.C, generator=g).to(torch.bfloat16)
    pos = torch.randint(0, 32, (sample_rows, 3), generator=g).float()
    cos, sin = rope_tables(pos, reference_dims(16), 10000.0)
    dt, n = _timed_repeat(lambda: ffn(attn(x, cos, sin)), min_seconds)
    step_s = dt * W.TOKENS / sample_rows
    return {"value": W.flops() / step_s / 1e12, "unit": "TFLOP/s",
            "cores": torch.get_num_threads(), "kind": "port", "s_per_step": step_s,
            "sample": (f"{sample_rows} of {W.TOKENS} rows (attention against all keys + SwiGLU "
                       f"FFN) x {n} repeats, {dt * n:.1f} s of CPU work, extrapolated "
                       f"linearly to every row")}


def cpu_baseline_run(args) -> dict | None:
    """The CPU arm of ``args.workload`` (None where it has none)."""
    if args.workload == "dit":
        return cpu_dit_estimate(args.cpu_rows, args.cpu_seconds)
    if args.workload == "ffn":
        return cpu_ffn_run(args.cpu_rows, args.cpu_seconds)
    if args.workload == "quant":
        return cpu_quant_run(args.cpu_rows, args.cpu_seconds)
    if args.workload == "attention":
        return cpu_attention_run([int(n) for n in args.attn_docs.split(",")], args.cpu_rows,
                                 args.cpu_seconds)
    if args.workload in ("refblock", "refblock-shims"):
        return cpu_refblock_run(args.cpu_rows, args.cpu_seconds)
    return None


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    vals = [cpu_baseline_run(args) for _ in range(max(args.steps, 1))]
    v = statistics.median([r["value"] for r in vals])
    r = vals[-1]
    unit = r["unit"]
    configs = {"dit": lambda: DiTWorkload.describe(args.gpus),
               "ffn": lambda: FFNWorkload.describe(args.gpus),
               "quant": lambda: QuantWorkload.describe(args.gpus),
               "attention": lambda: AttentionWorkload.describe(
                   args.gpus, [int(n) for n in args.attn_docs.split(",")]),
               "refblock": lambda: RefBlockWorkload.describe(args.gpus),
               "refblock-shims": lambda: RefShimsWorkload.describe(args.gpus)}
    dtypes = {"dit": "fp32 (NVFP4 operands decoded)", "ffn": "fp32 (NVFP4 operands decoded)",
              "quant": "fp32 -> e2m1 / e4m3", "attention": "fp32 (bf16 q|k|v)",
              "refblock": "fp32 (NVFP4 operands decoded)",
              "refblock-shims": "fp32 (NVFP4 operands decoded)"}
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": statistics.median([x["s_per_step"] for x in vals]) * 1e3,
        "ms_per_step_is": "extrapolated: the timed CPU sample scaled linearly to the whole step",
        "higher_is_better": True, "scaling": "strong" if args.workload == "dit" else "weak",
        "vs_baseline": None, "dtype": dtypes[args.workload],
        "data": "synthetic",
        "config": configs[args.workload](),
        "cpu_baseline": {"value": v, "unit": unit, "cores": r["cores"], "kind": r["kind"],
                         "sample": r["sample"]},
        "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU
def run_ours(args) -> None:
    import torch.distributed as dist

    from h3_engine_b200 import _lib
    from h3_engine_b200.parallel import init_distributed

    world, rank, local = init_distributed()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    if args.workload == "dit":
        wl = DiTWorkload(dev, world, rank)
    elif args.workload == "ffn":
        wl = FFNWorkload(dev, world, rank)
    elif args.workload == "refblock":
        wl = RefBlockWorkload(dev, world, rank)
    elif args.workload == "refblock-shims":
        wl = RefShimsWorkload(dev, world, rank)
    elif args.workload == "quant":
        wl = QuantWorkload(dev, world, rank)
    else:
        wl = AttentionWorkload(dev, world, rank, [int(n) for n in args.attn_docs.split(",")])
    for _ in range(args.warmup):
        wl.step()
    torch.cuda.synchronize()

    gemm_ev, attn_ev = [], []
    wl.set_timers(gemm_ev, attn_ev)
    launches0 = _lib.launch_count()
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            torch.cuda.nvtx.range_push("timed_step")     # ncu --nvtx-include "timed_step/"
            wl.step()
            torch.cuda.nvtx.range_pop()
        e1.record()
        torch.cuda.synchronize()
    barrier()
    launches = _lib.launch_count() - launches0
    wl.set_timers(None, None)
    ms = e0.elapsed_time(e1) / args.steps
    gemm_ms = sum(a.elapsed_time(b) for a, b in gemm_ev) / args.steps
    attn_list = [a.elapsed_time(b) for a, b in attn_ev]
    attn_ms = sum(attn_list) / args.steps
    err = _lib.device_error()
    if err:
        raise RuntimeError(f"device error {err} during the timed region")

    h2d, d2h = wl.e2e_setup()
    for _ in range(max(1, min(args.warmup, 2))):
        wl.e2e_step()
    torch.cuda.synchronize()
    barrier()
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(args.steps):
        wl.e2e_step()
    f1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = f0.elapsed_time(f1) / args.steps

    t = torch.tensor([ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = [float(v) for v in t.tolist()]

    extras = {}
    if world == 1 and wl.name == "dit" and not args.no_extras:
        extras["cuda_graph"] = graph_step_timing(wl, args.steps)
    if rank == 0 and not args.no_extras:
        extras["library_gemm_torch_scaled_mm"] = library_gemm_reference(
            dev, getattr(wl, "library_shapes", None))
        if wl.name in ("attention", "dit"):
            docs = ([b - a for a, b in zip(wl.cu[:-1], wl.cu[1:])] if wl.name == "attention"
                    else [b - a for a, b in zip(wl.cfg.cu_seqlens()[:-1], wl.cfg.cu_seqlens()[1:])])
            extras["library_attention_sdpa"] = library_attention_sdpa(
                dev, docs, copies=1 if wl.name == "attention" else 2)
        cpu = cpu_baseline_run(args) if world == 1 else None
        if cpu is not None:
            extras["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}

    if rank == 0:
        pk = peaks()
        gemm_tflops = wl.rank_gemm_flops / (gemm_ms * 1e-3) / 1e12 if gemm_ms else None
        if hasattr(wl, "roofline"):
            roof = wl.roofline(pk, args.steps, ms, sum(attn_list))
            if hasattr(wl, "unpack_rate"):
                extras["unpack"] = wl.unpack_rate(pk)
        elif attn_list:
            n_launch = len(attn_list)
            flops_launch = wl.rank_attn_flops * args.steps / n_launch
            achieved = flops_launch / (statistics.mean(attn_list) * 1e-3) / 1e12
            peak = pk["bf16_sustained"]
            roof = {"bound": "tensor", "kernel": "h3b::attn::k_fmha (bf16)", "achieved": achieved,
                    "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                    "peak_source": f"bf16_tflops_sustained of {pk['source']} MEASURED_PEAKS.json",
                    "traffic": (wl.attn_traffic if wl.name in ("dit", "refblock", "refblock-shims")
                                else ATTN_TRAFFIC_PER_TOKEN * wl.cu[-1]),
                    "per_launch_tflop": flops_launch / 1e12,
                    "launch_ms": statistics.mean(attn_list),
                    "share_of_step": attn_ms / ms}
        else:
            n_launch = len(gemm_ev)
            flops_launch = wl.rank_gemm_flops * args.steps / max(n_launch, 1)
            achieved = wl.rank_gemm_flops / (gemm_ms * 1e-3) / 1e12
            peak, source = fp4_peak(extras.get("library_gemm_torch_scaled_mm"), pk)
            roof = {"bound": "tensor", "kernel": "h3b::gemm::k_gemm_nvfp4", "achieved": achieved,
                    "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                    "peak_source": source,
                    "frac_of_nominal_9pf": achieved / NOMINAL_FP4_TFLOPS,
                    "traffic": TRAFFIC_BYTES["k_gemm_nvfp4"],
                    "per_launch_tflop": flops_launch / 1e12, "share_of_step": gemm_ms / ms}
        if hasattr(wl, "step_bytes"):           # memory-bound workload: GB/s
            unit, work, scale = "GB/s", wl.step_bytes, 1e9
            dtype = "bf16 in, e2m1 codes + e4m3 scales + fp32 global scale out"
        else:
            unit, work, scale = "TFLOP/s", wl.step_flops, 1e12
            dtype = "nvfp4 GEMMs (e2m1 x e4m3/16 x fp32 scale, fp32 accumulate) + bf16 attention"
        line = {
            "metric": METRIC,
            "value": work / (ms * 1e-3) / scale,
            "unit": unit,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if wl.name == "dit" else "weak",
            "vs_baseline": None,
            "dtype": dtype,
            "data": "synthetic (seeded random-init weights and latent of the configured shapes)",
            "config": wl.config,
            "e2e": {"value": work / (e2e_ms * 1e-3) / scale, "unit": unit,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "roofline": roof,
            "nvfp4_gemm_tflops_per_gpu": gemm_tflops,
            "nvfp4_gemm_frac_of_fp4_peak": (gemm_tflops / fp4_peak(
                extras.get("library_gemm_torch_scaled_mm"), pk)[0] if gemm_tflops else None),
            "fp4_peak_source": fp4_peak(extras.get("library_gemm_torch_scaled_mm"), pk)[1],
            "nvfp4_gemm_frac_of_nominal_9pf": (gemm_tflops / NOMINAL_FP4_TFLOPS
                                               if gemm_tflops else None),
            "gpu_launches": int(launches),
            "clocks": clk.summary(),
        }
        if wl.name == "dit":
            line["block_ms"] = ms / wl.cfg.blocks
            comm = wl.comm_summary(args.steps)
            if comm:
                line["collectives_rank0"] = comm
        line.update(extras)
        print(json.dumps(line), flush=True)
    if world > 1:
        if hasattr(wl, "layout"):
            wl.layout.close()
        dist.barrier()
        dist.destroy_process_group()


def graph_step_timing(wl, steps: int) -> dict:
    """The same denoising step replayed from one CUDA graph (one GPU)."""
    from h3_engine_b200.dit import GraphedSampler
    g = GraphedSampler(wl.sampler)
    x = wl.x
    for _ in range(2):
        x = g.step(x, wl.i % wl.sampler.steps)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for k in range(steps):
        x = g.step(x, (wl.i + k) % wl.sampler.steps)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    del g
    return {"ms_per_step": ms, "value": wl.step_flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s"}


def library_gemm_reference(dev, shapes: dict | None = None) -> dict | None:
    """torch._scaled_mm (cuBLASLt NVFP4, the reference's GEMM call at
    h3_inference/nvfp4.py:112-115) on 8192^3 and the GEMM shapes of the
    workloads, best of 3 runs of 10 back-to-back launches each: the measured
    dense-FP4 rate the GEMM fractions are quoted against.  Not part of the
    timed step."""
    try:
        from h3_engine_b200 import ops
        out = {}
        shapes = shapes or {"up": (FFN_TOKENS, FFN, HIDDEN), "down": (FFN_TOKENS, HIDDEN, FFN),
                            "square_8192": (8192, 8192, 8192)}
        for name, (M, N, K) in shapes.items():
            a = torch.randn(M, K, device=dev).to(torch.bfloat16)
            b = (torch.randn(N, K, device=dev) * 0.02).to(torch.bfloat16)
            qa, sa, _ = ops.quantize(a, mpad=ops.pad_m(M), gs=1.0)
            qb, sb, _ = ops.quantize(b, mpad=N, gs=1.0)
            a4, b4 = qa.view(torch.float4_e2m1fn_x2), qb.view(torch.float4_e2m1fn_x2).t()
            s1, s2 = sa.view(torch.float8_e4m3fn), sb.view(torch.float8_e4m3fn)
            for _ in range(3):
                torch._scaled_mm(a4, b4, s1, s2, out_dtype=torch.bfloat16)
            best = None
            for _ in range(3):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(10):
                    torch._scaled_mm(a4, b4, s1, s2, out_dtype=torch.bfloat16)
                e1.record()
                torch.cuda.synchronize()
                ms = e0.elapsed_time(e1) / 10
                best = ms if best is None else min(best, ms)
            mp = qa.shape[0]
            out[name] = {"shape": [M, N, K], "ms": best,
                         "tflops": 2.0 * mp * N * K / (best * 1e-3) / 1e12}
            del a, b, qa, qb
        return out
    except Exception as ex:  # pragma: no cover - library availability varies
        return {"unavailable": str(ex)[:160]}


def fp4_peak(lib: dict | None, pk: dict) -> tuple[float, str]:
    """Denominator of the NVFP4 GEMM fractions: the best cuBLASLt NVFP4 rate
    measured in this run (a dense-FP4 rate the library reaches on this GPU at
    this clock), else 4 x the measured bf16 burst rate."""
    rates = [v["tflops"] for v in (lib or {}).values() if isinstance(v, dict) and "tflops" in v]
    if rates:
        return max(rates), ("best torch._scaled_mm NVFP4 (cuBLASLt) rate measured in this run "
                            "over 8192^3 and the workload's GEMM shapes")
    return 4.0 * pk["bf16"], (f"4 x bf16_tflops (burst) of {pk['source']} MEASURED_PEAKS.json "
                              "(no library FP4 measurement in this run)")


NOMINAL_FP4_TFLOPS = 9000.0     # B200 dense FP4 (the 9 PFLOP/s figure the targets quote)


def library_attention_sdpa(dev, docs: list[int], heads: int = 24, head_dim: int = 128,
                           copies: int = 1) -> dict | None:
    """F.scaled_dot_product_attention (the reference's attention call,
    h3_inference/kernels/packed_self_attn.py:34-36) on the same packing, one
    call per document ([1, H, L, D] bf16, non-causal), with the cuDNN and the
    flash backends, best of 3 runs of 5; ``copies`` repeats the documents
    (the CFG pair)."""
    try:
        import torch.nn.functional as F
        from torch.nn.attention import SDPBackend, sdpa_kernel
        g = torch.Generator(device=dev).manual_seed(77)
        tensors = [[torch.randn(1, heads, n, head_dim, generator=g, device=dev).to(torch.bfloat16)
                    for _ in range(3)] for n in docs]
        flops = copies * sum(4 * heads * head_dim * n * n for n in docs)
        out = {}
        for name, be in (("cudnn", SDPBackend.CUDNN_ATTENTION), ("flash", SDPBackend.FLASH_ATTENTION)):
            try:
                with sdpa_kernel([be]):
                    def run():
                        for _ in range(copies):
                            for q, k, v in tensors:
                                F.scaled_dot_product_attention(q, k, v)
                    run()
                    torch.cuda.synchronize()
                    best = None
                    for _ in range(3):
                        e0 = torch.cuda.Event(enable_timing=True)
                        e1 = torch.cuda.Event(enable_timing=True)
                        e0.record()
                        for _ in range(5):
                            run()
                        e1.record()
                        torch.cuda.synchronize()
                        ms = e0.elapsed_time(e1) / 5
                        best = ms if best is None else min(best, ms)
                out[name] = {"ms": best, "tflops": flops / (best * 1e-3) / 1e12}
            except Exception as ex:   # backend not available for this shape / build
                out[name] = {"unavailable": str(ex)[:120]}
        del tensors
        return out
    except Exception as ex:  # pragma: no cover
        return {"unavailable": str(ex)[:160]}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["h3b", "reference"], default="h3b")
    ap.add_argument("--workload", choices=["dit", "ffn", "attention", "refblock", "refblock-shims",
                                           "quant"],
                    default="dit")
    ap.add_argument("--attn-docs", default="32760,1024",
                    help="document lengths of the attention workload (comma-separated)")
    ap.add_argument("--cpu-rows", type=int, default=256,
                    help="query rows (dit) / tokens (ffn) of the CPU sample")
    ap.add_argument("--cpu-seconds", type=float, default=CPU_SAMPLE_SECONDS,
                    help="CPU work per baseline sample (repeats of the row sample)")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the library GEMM comparison and the CPU baseline (profiling runs)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
