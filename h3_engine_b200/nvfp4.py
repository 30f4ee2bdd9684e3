"""Drop-in for ``h3_inference/nvfp4.py``: the same names, slots, return
values and error behaviour, computed by the sm_100a kernels in libh3b.so.

Differences, all additive:

* Three-level recipe.  Every quantized tensor carries an fp32 global scale
  (``global_scale``, a 1-element device tensor): ``gs = amax / (6 * 448)``
  over the tensor, E4M3 block scales per 16 values over that, E2M1 codes.
  The reference's two-level scheme is the special case ``gs = 1``
  (``_quantize(x, global_scale=1.0)``); a packed checkpoint without a global
  scale key loads with ``gs = 1``.
* ``_quantize`` returns the reference's ``(qdata, scale)`` pair; the pair also
  exposes ``.global_scale``.
* The GEMM is the tcgen05 block-scaled kernel, not ``torch._scaled_mm``.
There is no CPU or library fallback: without a CUDA device and the built
library every entry point raises.
"""
from __future__ import annotations

import os
from typing import Iterable

import torch
from torch import nn

from . import ops

FP4_BLOCK = 16          # h3_inference/nvfp4.py:9
FP4_MAX = 6.0           # h3_inference/nvfp4.py:10
M_ALIGN = 128           # h3_inference/nvfp4.py:12


def enabled() -> bool:
    """h3_inference/nvfp4.py:14-15."""
    return os.environ.get("H3_NVFP4") == "1" or os.environ.get("H3_KERNELS") == "1"


def _pad_m(m: int) -> int:
    """h3_inference/nvfp4.py:17-18."""
    return ((m + M_ALIGN - 1) // M_ALIGN) * M_ALIGN


class _QuantPair(tuple):
    """``(qdata, scale)`` that also carries the fp32 global scale."""

    global_scale: torch.Tensor

    def __new__(cls, qdata, scale, global_scale):
        obj = super().__new__(cls, (qdata, scale))
        obj.global_scale = global_scale
        return obj


def _check_input(x: torch.Tensor) -> None:
    if not x.is_cuda:
        raise RuntimeError("NVFP4 quantization runs on the GPU only (no CPU path)")
    if x.dtype != torch.bfloat16:
        raise TypeError(f"NVFP4 quantization expects bf16, got {x.dtype}")
    if x.shape[-1] % 64:
        raise ValueError(f"K = {x.shape[-1]} must be a multiple of 64")


@torch.no_grad()
def _quantize(x: torch.Tensor, global_scale: float | None = None):
    """bf16 ``(M, K)`` -> (packed fp4 ``(M, K//2)`` uint8, e4m3 scales ``(M, K//16)``).

    h3_inference/nvfp4.py:20-23.  Row-major scales as the reference returns
    them; ``.global_scale`` on the result.
    """
    _check_input(x)
    x2 = x.reshape(-1, x.shape[-1])
    M, K = x2.shape
    q, sf, gs = ops.quantize(x2, mpad=M, layout=ops.SF_ROWMAJOR, gs=global_scale)
    return _QuantPair(q, sf.view(M, K // FP4_BLOCK).view(torch.float8_e4m3fn), gs)


class _PadCache:
    """Per-(rows, cols) padded buffers, allocated once and reused
    (h3_inference/nvfp4.py:61-87)."""

    def __init__(self) -> None:
        self._data: dict[tuple, torch.Tensor] = {}
        self._scale: dict[tuple, torch.Tensor] = {}

    def data(self, rows: int, cols: int, device, dtype) -> torch.Tensor:
        key = (rows, cols, device, dtype)
        buf = self._data.get(key)
        if buf is None:
            buf = torch.zeros(rows, cols, device=device, dtype=dtype)
            self._data[key] = buf
        return buf

    def scale(self, rows: int, cols: int, device, dtype) -> torch.Tensor:
        key = (rows, cols, device, dtype)
        buf = self._scale.get(key)
        if buf is None:
            buf = torch.zeros(rows, cols, device=device, dtype=dtype)
            self._scale[key] = buf
        return buf

    def clear(self) -> None:
        self._data.clear()
        self._scale.clear()


_PAD = _PadCache()
# QuantizedActivation writes swizzled scales straight into its own buffers
# (the reference swizzles a copy of _PAD's row-major scales instead).
_ACT = _PadCache()


@torch.no_grad()
def _quantize_padded(x: torch.Tensor, mpad: int):
    """Quantize into the cached ``(mpad, ...)`` buffers; rows ``M..mpad-1`` are
    zero (h3_inference/nvfp4.py:25-42).  Scales are row-major like the
    reference's; ``QuantizedActivation`` uses the swizzled variant directly."""
    _check_input(x)
    xf = x.reshape(-1, x.shape[-1])
    m, k = xf.shape
    out = _PAD.data(mpad, k // 2, xf.device, torch.uint8)
    scale = _PAD.scale(mpad, k // FP4_BLOCK, xf.device, torch.uint8)
    _, _, gs = ops.quantize(xf, mpad=mpad, layout=ops.SF_ROWMAJOR, q_out=out,
                            sf_out=scale.view(-1))
    return _QuantPair(out, scale.view(torch.float8_e4m3fn), gs)


def _swizzle(scale: torch.Tensor) -> torch.Tensor:
    """Row-major ``(R, C)`` e4m3 scales -> the 128x4-tile layout consumed by the
    block-scaled GEMM (h3_inference/nvfp4.py:44-46; torchao ``to_blocked``
    semantics: rows padded to 128, columns to 4, returned flat)."""
    R, C = scale.shape
    rb, cb = -(-R // 128), -(-C // 4)
    p = torch.zeros(rb * 128, cb * 4, dtype=torch.uint8, device=scale.device)
    p[:R, :C] = scale.view(torch.uint8)
    t = p.view(rb, 128, cb, 4).permute(0, 2, 1, 3).reshape(rb, cb, 4, 32, 4)
    return t.permute(0, 1, 3, 2, 4).reshape(-1).view(torch.float8_e4m3fn)


def _unswizzle(blocked: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """Inverse of ``_swizzle``: u8 ``[rows, cols]`` row-major block scales from
    the flat 128x4-tile layout."""
    rb, cb = -(-rows // 128), -(-cols // 4)
    t = blocked.view(torch.uint8).reshape(rb, cb, 32, 4, 4).permute(0, 1, 3, 2, 4)
    t = t.reshape(rb, cb, 128, 4).permute(0, 2, 1, 3).reshape(rb * 128, cb * 4)
    return t[:rows, :cols]


class NVFP4Weight:
    """A quantized ``nn.Linear`` weight (h3_inference/nvfp4.py:48-59)."""

    __slots__ = ("qdata_t", "scale", "in_features", "out_features", "dtype", "global_scale")

    def __init__(self, weight: torch.Tensor):
        self.out_features, self.in_features = weight.shape
        self.dtype = weight.dtype
        w = weight.detach().to(torch.bfloat16).contiguous()
        _check_input(w)
        q, sf, gs = ops.quantize(w, mpad=_pad_m(self.out_features), layout=ops.SF_SWIZZLED)
        q = q[: self.out_features]
        self.qdata_t = q.view(torch.float4_e2m1fn_x2).t()      # (K/2, N) view, as the reference
        self.scale = sf.view(torch.float8_e4m3fn)              # swizzled
        self.global_scale = gs

    @classmethod
    def from_packed(cls, qdata: torch.Tensor, scale_swizzled: torch.Tensor,
                    out_features: int, in_features: int,
                    global_scale: torch.Tensor | float | None = None,
                    dtype: torch.dtype = torch.bfloat16) -> "NVFP4Weight":
        """Rebuild from packed checkpoint tensors (h3_inference/nvfp4.py:268-273)."""
        w = cls.__new__(cls)
        w.out_features, w.in_features, w.dtype = out_features, in_features, dtype
        w.qdata_t = qdata.view(torch.uint8).view(torch.float4_e2m1fn_x2).t()
        w.scale = scale_swizzled.view(torch.uint8).reshape(-1).view(torch.float8_e4m3fn)
        if global_scale is None:
            global_scale = 1.0
        if not isinstance(global_scale, torch.Tensor):
            global_scale = torch.tensor([float(global_scale)], dtype=torch.float32,
                                        device=qdata.device)
        w.global_scale = global_scale.reshape(1).to(torch.float32)
        return w

    @property
    def qdata(self) -> torch.Tensor:
        """u8 ``(N, K/2)``: the packed codes, K-major."""
        return self.qdata_t.t().view(torch.uint8)

    @property
    def scale_u8(self) -> torch.Tensor:
        return self.scale.view(torch.uint8)

    def nbytes(self) -> int:
        return self.qdata_t.numel() + self.scale.numel() * self.scale.element_size() + 4


class QuantizedActivation:
    """Quantize ``x`` once, multiply by any number of weights
    (h3_inference/nvfp4.py:89-115)."""

    __slots__ = ("qdata", "scale_blocked", "rows", "shape", "dtype", "global_scale")

    def __init__(self, x: torch.Tensor):
        _check_input(x)
        self.shape = x.shape
        self.dtype = x.dtype
        x2 = x.reshape(-1, x.shape[-1])
        self.rows = x2.shape[0]
        k = x2.shape[1]
        mpad = _pad_m(self.rows)
        # the RMSNorm + modulation shim leaves the NVFP4 form of its output on
        # the tensor (the kernel quantized exactly these bf16 values): reuse it
        # unless the tensor was written since
        pre = getattr(x, "_h3b_nvfp4", None)
        if pre is not None and pre[3] == x._version and pre[0].shape[0] == mpad:
            q, sf, gs = pre[:3]
            self.qdata = q.view(torch.float4_e2m1fn_x2)
            self.scale_blocked = sf.view(-1).view(torch.float8_e4m3fn)
            self.global_scale = gs
            return
        q = _ACT.data(mpad, k // 2, x2.device, torch.uint8)
        sf = _ACT.scale(mpad, k // FP4_BLOCK, x2.device, torch.uint8)
        _, _, gs = ops.quantize(x2, mpad=mpad, layout=ops.SF_SWIZZLED, q_out=q,
                                sf_out=sf.view(-1))
        self.qdata = q.view(torch.float4_e2m1fn_x2)
        self.scale_blocked = sf.view(-1).view(torch.float8_e4m3fn)
        self.global_scale = gs

    def mm(self, w: NVFP4Weight, out: torch.Tensor | None = None) -> torch.Tensor:
        k = self.shape[-1]
        if w.in_features != k:
            raise ValueError(f"in_features {w.in_features} != activation K {k}")
        y = ops.gemm(self.qdata.view(torch.uint8), self.scale_blocked.view(torch.uint8),
                     self.global_scale, self.rows, w.qdata, w.scale_u8, w.global_scale,
                     w.out_features, k, out=out)
        return y.reshape(*self.shape[:-1], w.out_features)


def nvfp4_linear(w: NVFP4Weight, x: torch.Tensor) -> torch.Tensor:
    """``x @ w.T`` in NVFP4 (h3_inference/nvfp4.py:118-120)."""
    return QuantizedActivation(x).mm(w)


def _block_linears(block: nn.Module) -> Iterable[tuple[nn.Module, str, nn.Linear]]:
    """h3_inference/nvfp4.py:122-130."""
    attn = block.attn
    yield attn, "to_q", attn.to_q
    yield attn, "to_k", attn.to_k
    yield attn, "to_v", attn.to_v
    yield attn.to_out, "0", attn.to_out[0]
    ff = block.ff
    yield ff.net[0], "proj", ff.net[0].proj
    yield ff.net, "2", ff.net[2]


class _QuantLinear(nn.Module):
    """h3_inference/nvfp4.py:132-144 (raises on a bias like the reference)."""

    def __init__(self, linear: nn.Linear):
        super().__init__()
        if linear.bias is not None:
            raise NotImplementedError("NVFP4 path does not carry a bias term")
        self.weight_nvfp4 = NVFP4Weight(linear.weight.data)
        self.in_features = linear.in_features
        self.out_features = linear.out_features
        self.calls = 0

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        self.calls += 1
        return nvfp4_linear(self.weight_nvfp4, x)


@torch.no_grad()
def quantize_blocks(model, self_check: bool = True) -> dict:
    """h3_inference/nvfp4.py:146-167."""
    if self_check and os.environ.get("H3_NVFP4_SELFCHECK") != "0":
        run_self_check(model)
    before = torch.cuda.memory_allocated()
    replaced = 0
    for block in model.transformer_blocks:
        for parent, attr, linear in list(_block_linears(block)):
            q = _QuantLinear(linear)
            if isinstance(parent, (nn.ModuleList, nn.Sequential)):
                parent[int(attr)] = q
            else:
                setattr(parent, attr, q)
            replaced += 1
    torch.cuda.empty_cache()
    after = torch.cuda.memory_allocated()
    return {
        "linears_quantized": replaced,
        "freed_gib": (before - after) / 1024**3,
        "resident_gib": after / 1024**3,
    }


@torch.no_grad()
def run_self_check(model, tol: float = 0.98) -> float:
    """cos >= 0.98 against bf16 F.linear (h3_inference/nvfp4.py:169-181)."""
    linear = model.transformer_blocks[0].attn.to_q
    w = linear.weight.data
    x = torch.randn(M_ALIGN * 2, w.shape[1], device=w.device, dtype=torch.bfloat16)
    ref = torch.nn.functional.linear(x, w.to(torch.bfloat16))
    got = nvfp4_linear(NVFP4Weight(w), x)
    cos = float(torch.nn.functional.cosine_similarity(ref.float().flatten(),
                                                      got.float().flatten(), dim=0))
    if cos < tol:
        raise RuntimeError(f"NVFP4 self-check failed: cos {cos:.5f} < {tol}. ")
    return cos


def _suffix_for(parent, attr: str, block) -> str:
    """h3_inference/nvfp4.py:284-293."""
    if parent is block.attn:
        return f"attn.{attr}.weight"
    if parent is block.attn.to_out:
        return f"attn.to_out.{attr}.weight"
    if parent is block.ff.net[0]:
        return f"ff.net.0.{attr}.weight"
    if parent is block.ff.net:
        return f"ff.net.{attr}.weight"
    raise KeyError(f"unmapped block Linear: {parent}.{attr}")


@torch.no_grad()
def load_quantized(model, path: str) -> dict:
    """Swap each block linear for one rebuilt from ``<key>_nvfp4`` /
    ``<key>_nvfp4_scale`` (+ optional ``<key>_nvfp4_global_scale``, absent ->
    1.0) tensors (h3_inference/nvfp4.py:231-282)."""
    import json
    from pathlib import Path

    from safetensors import safe_open

    folder = Path(path)
    index = next(folder.glob("*.safetensors.index.json"), None)
    if index is None:
        raise FileNotFoundError(f"no safetensors index under {folder}")
    weight_map = json.loads(index.read_text())["weight_map"]
    wanted: dict[str, tuple[str, str]] = {}
    for key in weight_map:
        if key.endswith("_nvfp4"):
            wanted[key[: -len("_nvfp4")]] = (key, key + "_scale")
    if not wanted:
        raise RuntimeError(f"{folder} carries no `_nvfp4` weights — is it the bf16 checkpoint?")

    device = next((p.device for p in model.parameters() if not p.is_meta), torch.device("cuda"))
    tensors: dict[str, torch.Tensor] = {}
    shards = {weight_map[k] for pair in wanted.values() for k in pair}
    shards |= {weight_map[k] for k in weight_map if k.endswith("_nvfp4_global_scale")}
    for shard in sorted(shards):
        with safe_open(str(folder / shard), framework="pt", device=str(device)) as f:
            for name in f.keys():
                if name.endswith(("_nvfp4", "_nvfp4_scale", "_nvfp4_global_scale")):
                    tensors[name] = f.get_tensor(name)

    replaced = 0
    for block_index, block in enumerate(model.transformer_blocks):
        for parent, attr, linear in list(_block_linears(block)):
            prefix = f"transformer_blocks.{block_index}." + _suffix_for(parent, attr, block)
            pair = wanted.get(prefix)
            if pair is None:
                raise KeyError(f"pre-quantized checkpoint is missing {prefix}_nvfp4")
            q = _QuantLinear.__new__(_QuantLinear)
            nn.Module.__init__(q)
            q.weight_nvfp4 = NVFP4Weight.from_packed(
                tensors[pair[0]], tensors[pair[1]], linear.out_features, linear.in_features,
                tensors.get(pair[0] + "_global_scale"))
            q.in_features, q.out_features = linear.in_features, linear.out_features
            q.calls = 0
            if isinstance(parent, (nn.ModuleList, nn.Sequential)):
                parent[int(attr)] = q
            else:
                setattr(parent, attr, q)
            replaced += 1
    torch.cuda.empty_cache()
    return {"linears_loaded": replaced, "resident_gib": torch.cuda.memory_allocated() / 1024**3}


@torch.no_grad()
def load_transformer_nvfp4(model_path: str, device: str = "cuda", model_cls=None):
    """h3_inference/nvfp4.py:184-229.  ``model_cls`` defaults to the
    reference's ``H3Transformer3DModel`` (imported lazily)."""
    import json
    from pathlib import Path

    from safetensors import safe_open

    if model_cls is None:
        from h3_inference.transformer.model import H3Transformer3DModel as model_cls
    folder = Path(model_path) / "transformer" if (Path(model_path) / "transformer").is_dir() \
        else Path(model_path)
    config = {k: v for k, v in json.loads((folder / "config.json").read_text()).items()
              if not k.startswith("_")}
    with torch.device("meta"):
        model = model_cls(**config)
    model.eval()
    model.requires_grad_(False)
    keep_fp32 = getattr(model_cls, "KEEP_IN_FP32", ())
    index = json.loads((folder / "model.safetensors.index.json").read_text())["weight_map"]
    state: dict[str, torch.Tensor] = {}
    for shard in sorted(set(index.values())):
        with safe_open(str(folder / shard), framework="pt", device=str(device)) as f:
            for name in f.keys():
                if name.endswith(("_nvfp4", "_nvfp4_scale", "_nvfp4_global_scale")):
                    continue
                dtype = torch.float32 if any(m in name for m in keep_fp32) else torch.bfloat16
                state[name] = f.get_tensor(name).to(dtype)
    model.load_state_dict(state, strict=False, assign=True)
    del state
    rope_theta = float(config.get("rope_theta", 10000.0))
    rope_freq_dim = int(config.get("rope_freq_dim", 16))
    model.rope.register_buffer(
        "inv_freq",
        1.0 / (rope_theta ** (torch.arange(0, 2 * rope_freq_dim, 2, dtype=torch.float32,
                                           device=device) / (2 * rope_freq_dim))),
        persistent=False,
    )
    summary = load_quantized(model, str(folder))
    stranded = [n for n, p in model.named_parameters() if p.is_meta]
    if stranded:
        raise RuntimeError(f"Parameters left on the meta device after NVFP4 load: {stranded[:8]}")
    return model, summary


def _fused_qkv(to_q, to_k, to_v):
    """The three packed weights concatenated along N (cached on ``to_q``);
    each keeps its own global scale through the GEMM's per-segment gsB."""
    cached = getattr(to_q, "_h3b_fused_qkv", None)
    ws = (to_q.weight_nvfp4, to_k.weight_nvfp4, to_v.weight_nvfp4)
    if cached is not None and cached[0] == tuple(id(w) for w in ws):
        return cached[1]
    n = ws[0].out_features
    if any(w.out_features != n or w.in_features != ws[0].in_features for w in ws) or n % 128:
        fused = None
    else:
        fused = (torch.cat([w.qdata for w in ws]), torch.cat([w.scale_u8 for w in ws]),
                 torch.cat([w.global_scale for w in ws]), n)
    try:
        object.__setattr__(to_q, "_h3b_fused_qkv", (tuple(id(w) for w in ws), fused))
    except Exception:
        pass
    return fused


def shared_qkv(to_q, to_k, to_v, x: torch.Tensor):
    """One activation quantization shared by q, k, v (h3_inference/nvfp4.py:295-302).
    Returns ``None`` unless all three are ``_QuantLinear``."""
    mods = (to_q, to_k, to_v)
    if not all(isinstance(m, _QuantLinear) for m in mods):
        return None
    act = QuantizedActivation(x)
    for m in mods:
        m.calls += 1
    fused = _fused_qkv(to_q, to_k, to_v)
    if fused is None:
        return tuple(act.mm(m.weight_nvfp4) for m in mods)
    qb, sfb, gsb, n = fused
    k = act.shape[-1]
    y = ops.gemm(act.qdata.view(torch.uint8), act.scale_blocked.view(torch.uint8),
                 act.global_scale, act.rows, qb, sfb, gsb, 3 * n, k, gsb_seg=n)
    y = y.reshape(*act.shape[:-1], 3 * n)
    return y[..., :n], y[..., n:2 * n], y[..., 2 * n:]


def report(model) -> str:
    """h3_inference/nvfp4.py:304-307."""
    served = sum(m.calls for m in model.modules() if isinstance(m, _QuantLinear))
    count = sum(1 for m in model.modules() if isinstance(m, _QuantLinear))
    return f"{count} NVFP4 linears, {served} calls served"
