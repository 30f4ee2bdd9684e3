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
    """Row-padded NVFP4 buffers reused across calls, one per (kind, rows,
    columns, device, dtype).  ``data`` / ``scale`` are the accessors of the
    reference's cache (h3_inference/nvfp4.py:61-87).  The buffers are left
    uninitialised: the quantizer writes every row up to the padded count,
    padding rows as zero codes and zero scales."""

    __slots__ = ("_store",)

    def __init__(self) -> None:
        self._store: dict[tuple, torch.Tensor] = {}

    def _get(self, kind: str, rows: int, cols: int, device, dtype) -> torch.Tensor:
        key = (kind, int(rows), int(cols), torch.device(device), dtype)
        buf = self._store.get(key)
        if buf is None:
            buf = self._store[key] = torch.empty((rows, cols), device=device, dtype=dtype)
        return buf

    def data(self, rows: int, cols: int, device, dtype) -> torch.Tensor:
        return self._get("codes", rows, cols, device, dtype)

    def scale(self, rows: int, cols: int, device, dtype) -> torch.Tensor:
        return self._get("scales", rows, cols, device, dtype)

    def clear(self) -> None:
        self._store.clear()


# _quantize_padded's buffers (row-major scales, as the reference returns them)
_PAD = _PadCache()
# QuantizedActivation's buffers: the quantizer writes the swizzled scales the
# GEMM reads straight into them, so no separate swizzle pass runs
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

    def mm(self, w, out: torch.Tensor | None = None) -> torch.Tensor:
        """``x @ w.T`` for this library's ``NVFP4Weight`` or a weight object of
        the reference's own ``nvfp4`` module (read with global scale 1)."""
        w = as_nvfp4_weight(w)
        k = self.shape[-1]
        if w.in_features != k:
            raise ValueError(f"in_features {w.in_features} != activation K {k}")
        y = ops.gemm(self.qdata.view(torch.uint8), self.scale_blocked.view(torch.uint8),
                     self.global_scale, self.rows, w.qdata, w.scale_u8, w.global_scale,
                     w.out_features, k, out=out)
        return y.reshape(*self.shape[:-1], w.out_features)


def as_nvfp4_weight(w) -> NVFP4Weight:
    """This library's ``NVFP4Weight`` for ``w``.  A weight built by the
    reference's own ``nvfp4`` module (slots ``qdata_t`` -- the packed codes
    viewed transposed -- and ``scale`` -- the swizzled e4m3 scales --, no
    global scale, h3_inference/nvfp4.py:48-59) is wrapped without copying,
    with the two-level scheme's global scale 1; the wrapper is cached on the
    object when it allows attributes, else rebuilt per call (a view)."""
    if isinstance(w, NVFP4Weight):
        return w
    cached = getattr(w, "_h3b_weight", None)
    if cached is not None and cached.qdata_t.data_ptr() == w.qdata_t.data_ptr():
        return cached
    n, k = int(w.out_features), int(w.in_features)
    packed = w.qdata_t.t().view(torch.uint8)
    gs = getattr(w, "global_scale", None)
    mine = NVFP4Weight.from_packed(packed, w.scale, n, k, gs, getattr(w, "dtype", torch.bfloat16))
    try:
        object.__setattr__(w, "_h3b_weight", mine)
    except (AttributeError, TypeError):
        pass
    return mine


def nvfp4_linear(w, x: torch.Tensor) -> torch.Tensor:
    """``x @ w.T`` in NVFP4 (h3_inference/nvfp4.py:118-120)."""
    return QuantizedActivation(x).mm(w)


# The six linears of a transformer block that the NVFP4 path replaces, as
# (parent module path inside the block, child name): q, k, v, the output
# projection, the fused SwiGLU [value | gate] projection and the down
# projection -- the set and order of h3_inference/nvfp4.py:122-130.
_BLOCK_LINEAR_SLOTS = (("attn", "to_q"), ("attn", "to_k"), ("attn", "to_v"),
                       ("attn.to_out", "0"), ("ff.net.0", "proj"), ("ff.net", "2"))


def _block_linears(block: nn.Module) -> Iterable[tuple[nn.Module, str, nn.Module]]:
    """(parent, child name, module) of each replaced linear of ``block``."""
    for path, name in _BLOCK_LINEAR_SLOTS:
        parent = block.get_submodule(path)
        yield parent, name, parent._modules[name]


def _suffix_for(parent, attr: str, block) -> str:
    """Checkpoint key suffix (``attn.to_q.weight``, ``ff.net.0.proj.weight``,
    ...) of the linear ``parent.<attr>`` of ``block`` (the key format of
    h3_inference/nvfp4.py:284-293)."""
    for path, name in _BLOCK_LINEAR_SLOTS:
        if name == attr and block.get_submodule(path) is parent:
            return f"{path}.{name}.weight"
    raise KeyError(f"unmapped block Linear: {parent}.{attr}")


def _set_child(parent: nn.Module, name: str, module: nn.Module) -> None:
    """Replace a registered child (a named attribute or a numbered slot of a
    ModuleList / Sequential alike: both live in ``_modules``)."""
    parent._modules[name] = module


class _QuantLinear(nn.Module):
    """An NVFP4 linear without bias (the reference's module,
    h3_inference/nvfp4.py:132-144: attributes ``weight_nvfp4``,
    ``in_features``, ``out_features`` and the ``calls`` counter; a linear
    with a bias is refused with the reference's error)."""

    def __init__(self, linear: nn.Linear):
        super().__init__()
        if linear.bias is not None:
            raise NotImplementedError("NVFP4 path does not carry a bias term")
        self._bind(NVFP4Weight(linear.weight.data))

    def _bind(self, weight: NVFP4Weight) -> None:
        self.weight_nvfp4 = weight
        self.in_features, self.out_features = weight.in_features, weight.out_features
        self.calls = 0

    @classmethod
    def from_weight(cls, weight: NVFP4Weight) -> "_QuantLinear":
        """Wrap an already-quantized weight (checkpoint loading)."""
        mod = cls.__new__(cls)
        nn.Module.__init__(mod)
        mod._bind(weight)
        return mod

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        self.calls += 1
        return QuantizedActivation(x).mm(self.weight_nvfp4)


def _is_quant_linear(m) -> bool:
    """True for this library's ``_QuantLinear`` and for any module carrying
    an NVFP4 weight object in ``weight_nvfp4`` (the reference's own
    ``_QuantLinear``)."""
    w = getattr(m, "weight_nvfp4", None)
    return w is not None and hasattr(w, "qdata_t") and hasattr(w, "scale")


_GIB = float(1 << 30)


@torch.no_grad()
def quantize_blocks(model, self_check: bool = True) -> dict:
    """Swap the six block linears of every transformer block for NVFP4
    ones, after the optional self-check (h3_inference/nvfp4.py:146-167; same
    return keys).  Only (parent, name) pairs are collected up front, so each
    bf16 weight is released as soon as its replacement is in place and
    ``freed_gib`` sees it."""
    if self_check and os.environ.get("H3_NVFP4_SELFCHECK") != "0":
        run_self_check(model)
    mem0 = torch.cuda.memory_allocated()
    slots = [(parent, name) for block in model.transformer_blocks
             for parent, name, _ in _block_linears(block)]
    for parent, name in slots:
        _set_child(parent, name, _QuantLinear(parent._modules[name]))
    torch.cuda.empty_cache()
    mem1 = torch.cuda.memory_allocated()
    return {"linears_quantized": len(slots), "freed_gib": (mem0 - mem1) / _GIB,
            "resident_gib": mem1 / _GIB}


@torch.no_grad()
def run_self_check(model, tol: float = 0.98) -> float:
    """Cosine similarity of the NVFP4 linear against the bf16 one on random
    rows, for the first block's query projection; raises below ``tol`` (the
    reference's check and message, h3_inference/nvfp4.py:169-181).  The row
    count is not a multiple of 128, so the padded-row path is exercised."""
    w = model.transformer_blocks[0].attn.to_q.weight.data
    gen = torch.Generator(device=w.device).manual_seed(0)
    x = torch.randn(3 * M_ALIGN - 37, w.shape[1], generator=gen, device=w.device)
    x = x.to(torch.bfloat16)
    ref = torch.nn.functional.linear(x, w.to(torch.bfloat16)).float().flatten()
    got = nvfp4_linear(NVFP4Weight(w), x).float().flatten()
    cos = float(torch.dot(ref, got) / (ref.norm() * got.norm()).clamp_min(1e-30))
    if cos < tol:
        raise RuntimeError(f"NVFP4 self-check failed: cos {cos:.5f} < {tol}. ")
    return cos


_PACKED_SUFFIXES = ("_nvfp4", "_nvfp4_scale", "_nvfp4_global_scale")


def _checkpoint_index(folder) -> dict[str, str]:
    """tensor name -> shard file, from the folder's safetensors index."""
    import json
    index = next(iter(sorted(folder.glob("*.safetensors.index.json"))), None)
    if index is None:
        raise FileNotFoundError(f"no safetensors index under {folder}")
    return json.loads(index.read_text())["weight_map"]


@torch.no_grad()
def load_quantized(model, path: str) -> dict:
    """Replace every block linear by an NVFP4 one rebuilt from the packed
    checkpoint tensors ``<key>_nvfp4`` (u8 [N, K/2]) and ``<key>_nvfp4_scale``
    (swizzled e4m3), plus the optional ``<key>_nvfp4_global_scale`` (absent:
    1.0, the two-level scheme).  Same keys, errors and return value as
    h3_inference/nvfp4.py:231-282.  Every linear is matched to its keys before
    any is replaced, then each shard is opened once for exactly the tensors
    it holds."""
    from pathlib import Path

    from safetensors import safe_open

    folder = Path(path)
    weight_map = _checkpoint_index(folder)
    packed = {k[: -len("_nvfp4")] for k in weight_map if k.endswith("_nvfp4")}
    if not packed:
        raise RuntimeError(f"{folder} carries no `_nvfp4` weights — is it the bf16 checkpoint?")
    plan = []
    for i, block in enumerate(model.transformer_blocks):
        for parent, name, lin in _block_linears(block):
            key = f"transformer_blocks.{i}." + _suffix_for(parent, name, block)
            if key not in packed:
                raise KeyError(f"pre-quantized checkpoint is missing {key}_nvfp4")
            plan.append((parent, name, key, lin.in_features, lin.out_features))
    by_shard: dict[str, list[str]] = {}
    for *_, key, _, _ in plan:
        for suffix in _PACKED_SUFFIXES:
            shard = weight_map.get(key + suffix)
            if shard is not None:
                by_shard.setdefault(shard, []).append(key + suffix)
    device = next((p.device for p in model.parameters() if not p.is_meta), torch.device("cuda"))
    tensors: dict[str, torch.Tensor] = {}
    for shard, names in sorted(by_shard.items()):
        with safe_open(str(folder / shard), framework="pt", device=str(device)) as f:
            for name in names:
                tensors[name] = f.get_tensor(name)
    for parent, name, key, k, n in plan:
        weight = NVFP4Weight.from_packed(tensors[key + "_nvfp4"], tensors[key + "_nvfp4_scale"],
                                         n, k, tensors.get(key + "_nvfp4_global_scale"))
        _set_child(parent, name, _QuantLinear.from_weight(weight))
    torch.cuda.empty_cache()
    return {"linears_loaded": len(plan), "resident_gib": torch.cuda.memory_allocated() / _GIB}


@torch.no_grad()
def load_transformer_nvfp4(model_path: str, device: str = "cuda", model_cls=None):
    """Build the transformer from a packed checkpoint folder: the model on the
    meta device, its dense tensors loaded in place (fp32 for the model's
    ``KEEP_IN_FP32`` names, bf16 otherwise), the RoPE frequencies rebuilt from
    the config, then ``load_quantized`` for the block linears; fails if any
    parameter stays on the meta device (h3_inference/nvfp4.py:184-229).
    ``model_cls`` defaults to the reference's ``H3Transformer3DModel``
    (imported lazily)."""
    import json
    from pathlib import Path

    from safetensors import safe_open

    if model_cls is None:
        from h3_inference.transformer.model import H3Transformer3DModel as model_cls
    root = Path(model_path)
    folder = root / "transformer" if (root / "transformer").is_dir() else root
    raw = json.loads((folder / "config.json").read_text())
    config = {k: v for k, v in raw.items() if not k.startswith("_")}
    with torch.device("meta"):
        model = model_cls(**config)
    model.eval()
    model.requires_grad_(False)

    fp32_names = tuple(getattr(model_cls, "KEEP_IN_FP32", ()))
    weight_map = json.loads((folder / "model.safetensors.index.json").read_text())["weight_map"]
    dense: dict[str, torch.Tensor] = {}
    for shard in sorted(set(weight_map.values())):
        with safe_open(str(folder / shard), framework="pt", device=str(device)) as f:
            for name in f.keys():
                if name.endswith(_PACKED_SUFFIXES):
                    continue
                keep = any(tag in name for tag in fp32_names)
                dense[name] = f.get_tensor(name).to(torch.float32 if keep else torch.bfloat16)
    model.load_state_dict(dense, strict=False, assign=True)
    dense.clear()

    theta = float(config.get("rope_theta", 10000.0))
    half = int(config.get("rope_freq_dim", 16))
    exponents = torch.arange(half, dtype=torch.float32, device=device) / half
    model.rope.register_buffer("inv_freq", 1.0 / torch.pow(theta, exponents), persistent=False)

    summary = load_quantized(model, str(folder))
    left = [n for n, p in model.named_parameters() if p.is_meta]
    if left:
        raise RuntimeError(f"Parameters left on the meta device after NVFP4 load: {left[:8]}")
    return model, summary


def _fused_qkv(to_q, to_k, to_v):
    """The three packed weights concatenated along N (cached on ``to_q``);
    each keeps its own global scale through the GEMM's per-segment gsB."""
    ws = tuple(as_nvfp4_weight(m.weight_nvfp4) for m in (to_q, to_k, to_v))
    tag = tuple(w.qdata_t.data_ptr() for w in ws)
    cached = getattr(to_q, "_h3b_fused_qkv", None)
    if cached is not None and cached[0] == tag:
        return cached[1]
    n = ws[0].out_features
    if any(w.out_features != n or w.in_features != ws[0].in_features for w in ws) or n % 128:
        fused = None
    else:
        fused = (torch.cat([w.qdata for w in ws]), torch.cat([w.scale_u8 for w in ws]),
                 torch.cat([w.global_scale for w in ws]), n)
    try:
        object.__setattr__(to_q, "_h3b_fused_qkv", (tag, fused))
    except (AttributeError, TypeError):
        pass
    return fused


def shared_qkv(to_q, to_k, to_v, x: torch.Tensor):
    """q, k and v projections from ONE quantization of ``x``
    (h3_inference/nvfp4.py:295-302): None unless all three modules carry an
    NVFP4 weight -- this library's ``_QuantLinear`` or the reference's own --
    else one N-concatenated GEMM (or three when the shapes do not fuse)."""
    mods = (to_q, to_k, to_v)
    if not all(_is_quant_linear(m) for m in mods):
        return None
    act = QuantizedActivation(x)
    for m in mods:
        m.calls = getattr(m, "calls", 0) + 1
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
    """Count of NVFP4 linears and of the calls they served
    (h3_inference/nvfp4.py:304-307)."""
    calls = [m.calls for m in model.modules() if isinstance(m, _QuantLinear)]
    return f"{len(calls)} NVFP4 linears, {sum(calls)} calls served"
