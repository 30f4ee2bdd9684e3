"""Benchmark of the NVFP4 DiT hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl h3b|reference]

Workload (one step): the DiT FFN sub-block on 32768 tokens x hidden 3072,
FFN 12288, seed 2: RMSNorm (eps 1e-6) -> NVFP4 GEMM up (+b1, GELU-tanh) ->
NVFP4 re-quantization -> NVFP4 GEMM down (+b2) -> residual add, bf16 out.
Synthetic inputs of the configured shapes/distributions (no dataset).

value  = whole-job NVFP4 GEMM throughput: N * 4 * T * d * f flops / step time
         (max over ranks), TFLOP/s; ms_per_step is the sub-block latency.
e2e    = the same metric through FFNBlock.__call__ with the step's input
         copied from pinned host memory and the output copied back, every step.
Multi-GPU: one process per GPU (torchrun), each rank runs its own 32768
tokens with replicated weights -- token sharding with no collective on the
data path, so scaling is weak.
--impl reference: the reference's NVFP4 path cannot run on a CPU (the
quantizer is in the absent maiku package), so the timed CPU implementation
is the torch-CPU port of the recipe with the reference's own decode
(oracle/cpu_torch.py) on a bounded token sample, all host threads.
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
TOKENS, HIDDEN, FFN = 32768, 3072, 12288
EPS = 1e-6
SEED = 2
WORKLOAD = ("DiT FFN sub-block (seed 2): RMSNorm -> NVFP4 GEMM up 3072->12288 (+bias, GELU-tanh) "
            "-> NVFP4 re-quant -> NVFP4 GEMM down 12288->3072 (+bias) -> residual")
# Per-launch DRAM traffic of the dominant kernel (the NVFP4 GEMM), from the
# committed ncu summary profiles/gemm_nvfp4_ffn.md (dram__bytes_read.sum +
# dram__bytes_write.sum, mean of the up and down projections).  None until captured.
GEMM_TRAFFIC_BYTES = None


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
        self.lines = []
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
        for ln in getattr(self, "lines", []):
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


# ----------------------------------------------------------------------------- inputs
def make_weights(dev):
    g = torch.Generator(device="cpu").manual_seed(SEED)
    w1 = (torch.randn(FFN, HIDDEN, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(HIDDEN, FFN, generator=g) * 0.02).to(torch.bfloat16)
    b1 = (torch.randn(FFN, generator=g) * 0.01).to(torch.bfloat16)
    b2 = (torch.randn(HIDDEN, generator=g) * 0.01).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(HIDDEN, generator=g)).to(torch.bfloat16)
    return [t.to(dev) for t in (w1, b1, w2, b2, gamma)]


def make_tokens(rank: int, dev, n: int = TOKENS):
    g = torch.Generator(device=dev).manual_seed(SEED * 1000 + rank)
    return torch.randn(n, HIDDEN, generator=g, device=dev).to(torch.bfloat16)


def gemm_flops(tokens: int) -> float:
    return 4.0 * tokens * HIDDEN * FFN


# ----------------------------------------------------------------------------- CPU
def cpu_sample_run(steps: int, warmup: int, sample_tokens: int) -> dict:
    """Times the torch-CPU port on a bounded token sample; returns TFLOP/s."""
    from oracle.cpu_torch import FFNBlockCPU

    torch.set_num_threads(os.cpu_count() or 1)
    w1, b1, w2, b2, gamma = make_weights("cpu")
    blk = FFNBlockCPU(w1, b1, w2, b2, gamma, EPS)
    g = torch.Generator().manual_seed(SEED * 1000)
    x = torch.randn(sample_tokens, HIDDEN, generator=g).to(torch.bfloat16)
    for _ in range(warmup):
        blk(x)
    t0 = time.perf_counter()
    for _ in range(steps):
        blk(x)
    dt = (time.perf_counter() - t0) / max(steps, 1)
    return {"value": gemm_flops(sample_tokens) / dt / 1e12, "unit": "TFLOP/s",
            "cores": torch.get_num_threads(), "kind": "port", "s_per_step": dt,
            "sample": f"{sample_tokens} of {TOKENS} tokens per step (same weights, seed 2)"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    r = cpu_sample_run(max(args.steps, 1), max(args.warmup, 0), args.cpu_tokens)
    line = {
        "impl": "reference", "metric": METRIC, "value": r["value"], "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": r["s_per_step"] * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32 (NVFP4 operands decoded)", "data": "synthetic",
        "config": {"workload": WORKLOAD + f" [CPU sample: {args.cpu_tokens} tokens]",
                   "tokens": args.cpu_tokens, "hidden": HIDDEN, "ffn": FFN},
        "cpu_baseline": {"value": r["value"], "unit": "TFLOP/s", "cores": r["cores"],
                         "kind": r["kind"], "sample": r["sample"]},
        "e2e": {"value": r["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU
def run_ours(args) -> None:
    import torch.distributed as dist

    from h3_engine_b200 import _lib
    from h3_engine_b200.blocks import FFNBlock

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    w1, b1, w2, b2, gamma = make_weights(dev)
    blk = FFNBlock(w1, b1, w2, b2, gamma, EPS)
    tokens = args.tokens
    x = make_tokens(rank, dev, tokens)
    y = torch.empty_like(x)
    flops = gemm_flops(tokens)

    for _ in range(args.warmup):
        blk(x, out=y)
    torch.cuda.synchronize()

    blk.gemm_events = []
    launches0 = _lib.launch_count()
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            blk(x, out=y)
        e1.record()
        torch.cuda.synchronize()
    barrier()
    launches = _lib.launch_count() - launches0
    ms = e0.elapsed_time(e1) / args.steps
    gemm_ms = [a.elapsed_time(b) for a, b in blk.gemm_events]
    blk.gemm_events = None
    err = _lib.device_error()
    if err:
        raise RuntimeError(f"device error {err} during the timed region")

    # e2e through the public call: pinned host in -> block -> pinned host out
    x_h = x.cpu().pin_memory()
    y_h = torch.empty_like(x_h).pin_memory()
    x_d = torch.empty_like(x)
    for _ in range(max(1, min(args.warmup, 2))):
        x_d.copy_(x_h, non_blocking=True)
        blk(x_d, out=y)
        y_h.copy_(y, non_blocking=True)
    torch.cuda.synchronize()
    barrier()
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(args.steps):
        x_d.copy_(x_h, non_blocking=True)
        blk(x_d, out=y)
        y_h.copy_(y, non_blocking=True)
    f1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = f0.elapsed_time(f1) / args.steps

    t = torch.tensor([ms, e2e_ms, statistics.mean(gemm_ms)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms, gemm_avg = [float(v) for v in t.tolist()]

    library = None
    cpu = None
    if rank == 0 and not args.no_extras:
        library = library_gemm_reference(dev)
    if rank == 0 and world == 1 and not args.no_extras:
        cpu = cpu_sample_run(1, 0, args.cpu_tokens)

    if rank == 0:
        pk = peaks()
        fp4_peak = 4.0 * pk["bf16_sustained"]
        achieved = (flops / 2) / (gemm_avg * 1e-3) / 1e12
        line = {
            "metric": METRIC,
            "value": world * flops / (ms * 1e-3) / 1e12,
            "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "nvfp4 (e2m1 x e4m3/16 x fp32), fp32 accumulate, bf16 out",
            "data": "synthetic (seeded, shapes/distributions of the FFN sub-block config)",
            "config": {"workload": WORKLOAD, "tokens_per_gpu": tokens, "hidden": HIDDEN,
                       "ffn": FFN, "parallelism": f"token-sharded x{world}, weights replicated",
                       "l2": "working set ~1.3 GB per step > 126 MB L2 (no flush needed)"},
            "e2e": {"value": world * flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": x.numel() * 2, "d2h_bytes_per_step": y.numel() * 2},
            "roofline": {"bound": "tensor", "kernel": "h3b::gemm::k_gemm_nvfp4",
                         "achieved": achieved, "peak": fp4_peak, "unit": "TFLOP/s",
                         "frac": achieved / fp4_peak,
                         "peak_source": f"4 x bf16_tflops_sustained of {pk['source']} "
                                        "MEASURED_PEAKS.json (B200 dense FP4 = 4x bf16 rate)",
                         "traffic": GEMM_TRAFFIC_BYTES,
                         "per_launch_gflop": flops / 2 / 1e9, "launch_ms": gemm_avg},
            "gpu_launches": int(launches),
            "clocks": clk.summary(),
        }
        if library is not None:
            line["library_gemm_torch_scaled_mm"] = library
        if cpu is not None:
            line["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def library_gemm_reference(dev) -> dict | None:
    """torch._scaled_mm (cuBLASLt NVFP4, the reference's GEMM call) on the
    same two GEMM shapes, for context; not part of the timed step."""
    try:
        from h3_engine_b200 import ops
        out = {}
        for name, (M, N, K) in {"up": (TOKENS, FFN, HIDDEN), "down": (TOKENS, HIDDEN, FFN)}.items():
            a = torch.randn(M, K, device=dev).to(torch.bfloat16)
            b = (torch.randn(N, K, device=dev) * 0.02).to(torch.bfloat16)
            qa, sa, _ = ops.quantize(a, mpad=M, gs=1.0)
            qb, sb, _ = ops.quantize(b, mpad=N, gs=1.0)
            a4, b4 = qa.view(torch.float4_e2m1fn_x2), qb.view(torch.float4_e2m1fn_x2).t()
            s1, s2 = sa.view(torch.float8_e4m3fn), sb.view(torch.float8_e4m3fn)
            for _ in range(3):
                torch._scaled_mm(a4, b4, s1, s2, out_dtype=torch.bfloat16)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(10):
                torch._scaled_mm(a4, b4, s1, s2, out_dtype=torch.bfloat16)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / 10
            out[name] = {"ms": ms, "tflops": 2.0 * M * N * K / (ms * 1e-3) / 1e12}
            del a, b, qa, qb
        return out
    except Exception as ex:  # pragma: no cover - library availability varies
        return {"unavailable": str(ex)[:160]}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["h3b", "reference"], default="h3b")
    ap.add_argument("--tokens", type=int, default=TOKENS,
                    help="tokens per GPU (default: the configured 32768; smaller for ncu captures)")
    ap.add_argument("--cpu-tokens", type=int, default=1024,
                    help="token sample for the CPU baseline")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the library GEMM comparison and the CPU baseline (profiling runs)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
