"""Dispatch surface of the row shims (h3_inference/kernels/_dispatch.py:1-65).

``MISS``, ``enabled(flag)``, ``armed_counts()`` and ``try_call(name, *args)``
behave as the reference's: a flag is on when it or ``H3_KERNELS`` is "1"
(counted per flag), and ``try_call`` returns the result of a covered call or
``MISS``.  Here ``try_call`` is answered by this library instead of the
reference's un-vendored plug-in package, so the reference's own shim modules
reach these kernels once its plug-in import resolves to this module::

    import sys, types
    from h3_engine_b200.kernels import _dispatch
    sys.modules["maiku"] = types.ModuleType("maiku")
    sys.modules["maiku.dispatch"] = _dispatch

Names answered (the strings the reference's shims pass):
``rope``, ``norm_rope_h3``, ``norm_modulate_h3``, ``ada_modulate_gather``,
``gate_residual_gather`` (elementwise_norm_rope.py), ``attention``
(packed_self_attn.py), ``qkv_projection``, ``out_projection``, ``ffn``
(ffn_qkvo_gemms.py).  The library's own blocks fuse the modulation gather
into the RMSNorm -> NVFP4 kernel and the gate + residual into the GEMM
epilogue; the two gather kernels serve the reference's block, which calls
them as separate rows.

A call whose arguments the kernels do not take (CPU tensors, an attention
mask, head_dim other than 128 for attention, rotary widths whose half is not
a multiple of 8, ...) is MISS, on which the shims run the reference's stock
torch expression, as the reference does.  A covered call never falls back:
a missing libh3b.so or a failing launch raises.  ``miss_counts()`` reports
the MISSes per name (of ``try_call`` and of the armed shims).
"""
from __future__ import annotations

import os
from typing import Any


class _Miss:
    __slots__ = ()

    def __repr__(self) -> str:
        return "MISS"

    def __bool__(self) -> bool:
        return False


MISS: Any = _Miss()

_ARMED: dict[str, int] = {}
_MISSED: dict[str, int] = {}


def enabled(flag: str) -> bool:
    on = os.environ.get(flag) == "1" or os.environ.get("H3_KERNELS") == "1"
    if on:
        _ARMED[flag] = _ARMED.get(flag, 0) + 1
    return on


def armed_counts(reset: bool = False) -> dict[str, int]:
    out = dict(_ARMED)
    if reset:
        _ARMED.clear()
    return out


def miss_counts(reset: bool = False) -> dict[str, int]:
    out = dict(_MISSED)
    if reset:
        _MISSED.clear()
    return out


_TABLE: dict | None = None


def _table() -> dict:
    global _TABLE
    if _TABLE is not None:
        return _TABLE
    from h3_engine_b200.kernels import elementwise_norm_rope as ew
    from h3_engine_b200.kernels import ffn_qkvo_gemms as gm
    from h3_engine_b200.kernels import packed_self_attn as at
    _TABLE = {
        "rope": lambda x, cos, sin: ew.rope_kernel(x, None, 0.0, cos, sin),
        "norm_rope_h3": ew.rope_kernel,
        "norm_modulate_h3": ew.norm_modulate_kernel,
        "ada_modulate_gather": ew.ada_modulate_kernel,
        "gate_residual_gather": ew.gate_residual_kernel,
        "attention": at.attention_kernel_flat,
        "qkv_projection": gm.qkv_kernel,
        "out_projection": gm.out_kernel,
        "ffn": gm.ffn_kernel,
    }
    return _TABLE


def note_miss(name: str) -> None:
    """Count an armed call the kernels did not take (the shims call this too)."""
    _MISSED[name] = _MISSED.get(name, 0) + 1


def try_call(name: str, *args, **kwargs):
    fn = _table().get(name)
    out = MISS if fn is None else fn(*args, **kwargs)
    if out is MISS:
        note_miss(name)
    return out


def maiku_status() -> str:
    """The reference reports its plug-in's state here; this is the library's."""
    try:
        from h3_engine_b200 import _lib
        _lib.lib()
        return f"loaded: {_lib.LIB_PATH}"
    except Exception as exc:  # reported, not swallowed: try_call raises the same error
        return f"unavailable: {type(exc).__name__}: {exc}"
