"""Pre-quantize a bf16 safetensors transformer checkpoint to packed NVFP4.

Drop-in for h3_inference/quantize_ckpt.py:17-92 (same selection of weights,
same key names, same shard / index / metadata layout), on this package's
quantizer:

* every ``transformer_blocks.*`` weight ending in one of ``QUANT_SUFFIXES``
  becomes ``<key>_nvfp4`` (u8 ``[N, K/2]``, two E2M1 codes per byte, low
  nibble = even K index) and ``<key>_nvfp4_scale`` (u8 view of the e4m3 block
  scales in the 128x4-tile layout);
* new here: ``<key>_nvfp4_global_scale`` (fp32 ``[1]``, amax / 2688), read by
  ``nvfp4.load_quantized`` (absent -> 1.0, the reference's two-level scheme);
* every other tensor is copied through; shards are renamed
  ``model-XXXXX-of-YYYYY.safetensors`` with metadata ``h3_quant: nvfp4`` and a
  fresh ``model.safetensors.index.json``; ``config.json`` is copied.

    python -m h3_engine_b200.quantize_ckpt --src <bf16 dir> --dst <out dir> [--verify]

``--verify`` runs one GEMM per weight through the stored operands against the
bf16 ``F.linear`` and fails below cosine 0.98 (the reference's bar,
h3_inference/quantize_ckpt.py:95-114).
"""
from __future__ import annotations

import argparse
import json
import shutil
import sys
import time
from dataclasses import dataclass, field
from pathlib import Path

import torch

QUANT_SUFFIXES = (
    ".attn.to_q.weight",
    ".attn.to_k.weight",
    ".attn.to_v.weight",
    ".attn.to_out.0.weight",
    ".ff.net.0.proj.weight",
    ".ff.net.2.weight",
)
COS_BAR = 0.98


def is_quantizable(key: str) -> bool:
    """A transformer-block linear weight the hot path runs in NVFP4."""
    return key.startswith("transformer_blocks.") and key.endswith(QUANT_SUFFIXES)


@torch.no_grad()
def quantize_weight(w: torch.Tensor, device: str = "cuda"):
    """bf16 ``[N, K]`` -> (u8 ``[N, K/2]``, u8 blocked scales, fp32 ``[1]``
    global scale), all on the CPU."""
    from .nvfp4 import NVFP4Weight

    nw = NVFP4Weight(w.to(device=device, dtype=torch.bfloat16).contiguous())
    return nw.qdata.cpu(), nw.scale_u8.cpu(), nw.global_scale.reshape(1).float().cpu()


@torch.no_grad()
def verify_weight(w: torch.Tensor, qdata, scale, gs, device: str = "cuda") -> float:
    """Cosine between ``F.linear(x, w)`` and the GEMM through the stored
    operands on 128 random rows."""
    from .nvfp4 import NVFP4Weight, QuantizedActivation

    wb = w.to(device=device, dtype=torch.bfloat16)
    n, k = wb.shape
    g = torch.Generator(device=device).manual_seed(0)
    x = torch.randn(128, k, device=device, generator=g).to(torch.bfloat16)
    stored = NVFP4Weight.from_packed(qdata.to(device), scale.to(device), n, k, gs.to(device))
    got = QuantizedActivation(x).mm(stored)
    ref = torch.nn.functional.linear(x, wb)
    return float(torch.nn.functional.cosine_similarity(ref.float().flatten(),
                                                       got.float().flatten(), dim=0))


def _source_shards(src: Path) -> list[Path]:
    index = next(src.glob("*.safetensors.index.json"), None)
    if index is not None:
        names = sorted(set(json.loads(index.read_text())["weight_map"].values()))
        return [src / n for n in names]
    return sorted(src.glob("*.safetensors"))


@dataclass
class Summary:
    quantized: int = 0
    copied: int = 0
    bytes_in: int = 0
    bytes_out: int = 0
    worst_cos: float = 1.0
    weight_map: dict = field(default_factory=dict)


@torch.no_grad()
def run(src: str, dst: str, verify: bool = False, device: str = "cuda", log=print) -> int:
    """Quantize every shard of ``src`` into ``dst``; 0 on success, 1 when a
    verified weight falls below the cosine bar."""
    from safetensors import safe_open
    from safetensors.torch import save_file

    src_dir, dst_dir = Path(src), Path(dst)
    dst_dir.mkdir(parents=True, exist_ok=True)
    shards = _source_shards(src_dir)
    if not shards:
        raise FileNotFoundError(f"no safetensors shards under {src_dir}")
    s = Summary()
    t0 = time.perf_counter()
    for i, shard in enumerate(shards, 1):
        out: dict[str, torch.Tensor] = {}
        with safe_open(str(shard), framework="pt", device="cpu") as f:
            for key in f.keys():
                t = f.get_tensor(key)
                s.bytes_in += t.numel() * t.element_size()
                if not is_quantizable(key):
                    out[key] = t
                    s.copied += 1
                    continue
                q, sc, gs = quantize_weight(t, device)
                out[key + "_nvfp4"], out[key + "_nvfp4_scale"] = q, sc
                out[key + "_nvfp4_global_scale"] = gs
                s.quantized += 1
                if verify:
                    s.worst_cos = min(s.worst_cos, verify_weight(t, q, sc, gs, device))
        name = f"model-{i:05d}-of-{len(shards):05d}.safetensors"
        shard_bytes = sum(t.numel() * t.element_size() for t in out.values())
        s.bytes_out += shard_bytes
        s.weight_map.update({k: name for k in out})
        save_file(out, str(dst_dir / name), metadata={"format": "pt", "h3_quant": "nvfp4"})
        log(f"  [{i}/{len(shards)}] {name}  {shard_bytes / 2**30:.2f} GiB")
    (dst_dir / "model.safetensors.index.json").write_text(json.dumps(
        {"metadata": {"total_size": s.bytes_out, "h3_quant": "nvfp4"},
         "weight_map": s.weight_map}, indent=2))
    if (src_dir / "config.json").exists():
        shutil.copy(src_dir / "config.json", dst_dir / "config.json")
    log(f"{s.quantized} weights quantized, {s.copied} copied through unchanged; "
        f"{s.bytes_in / 2**30:.2f} GiB -> {s.bytes_out / 2**30:.2f} GiB "
        f"in {time.perf_counter() - t0:.0f} s")
    if verify:
        log(f"worst per-weight cos vs bf16: {s.worst_cos:.5f}")
        if s.worst_cos < COS_BAR:
            log("  FAILED")
            return 1
    return 0


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="h3_engine_b200.quantize_ckpt", description=__doc__,
                                formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--src", required=True, help="bf16 transformer checkpoint directory")
    p.add_argument("--dst", required=True, help="output directory")
    p.add_argument("--verify", action="store_true",
                   help=f"one GEMM per weight through the stored operands (cos >= {COS_BAR})")
    a = p.parse_args(argv)
    return run(a.src, a.dst, a.verify)


if __name__ == "__main__":
    sys.exit(main())
