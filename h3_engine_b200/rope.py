"""Rotary tables for the packed multimodal sequence.

``rope_tables`` builds the fp32 (cos, sin) tables that the qk-norm + RoPE
kernel consumes, in the layout of the reference's ``H3RotaryPosEmbed``
(h3_inference/transformer/model.py:23-38): the first half of the rotary dims
holds the angles of the t axis, then h, then w; the second half repeats them
(rotate-half pairs j and j + R/2 share an angle).  The reference shares one
``inv_freq`` of length ``rope_freq_dim`` across the three axes
(``axis_dims = (2*rope_freq_dim,)*3``); the GELU/bias configuration splits
head_dim 128 as 44/42/42 with a per-axis ``inv_freq = theta^(-2i/d_axis)``.
Computed once per forward and shared by every block.
"""
from __future__ import annotations

import torch


def axis_inv_freq(dims: tuple[int, ...], theta: float, device) -> list[torch.Tensor]:
    return [1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float32, device=device) / d))
            for d in dims]


def rope_tables(position_ids: torch.Tensor, dims: tuple[int, ...] = (44, 42, 42),
                theta: float = 10000.0) -> tuple[torch.Tensor, torch.Tensor]:
    """``position_ids``: (T, 3) -> fp32 ``cos``, ``sin`` of shape (T, sum(dims))."""
    pos = position_ids.to(torch.float32)
    invs = axis_inv_freq(dims, theta, pos.device)
    freqs = torch.cat([pos[:, a:a + 1] * inv[None, :] for a, inv in enumerate(invs)], dim=-1)
    freqs = torch.cat((freqs, freqs), dim=-1)
    return freqs.cos(), freqs.sin()


def reference_dims(rope_freq_dim: int = 16) -> tuple[int, int, int]:
    """Axis widths that reproduce the reference's shared-inv_freq layout."""
    return (2 * rope_freq_dim,) * 3


def packed_positions(grid_thw: tuple[int, int, int], audio_tokens: int,
                     device=None) -> torch.Tensor:
    """(T, 3) positions of a packed [video (t, h, w grid) | audio] sequence:
    video tokens carry their (t, h, w) grid coordinates, audio tokens a 1-D
    position on the t axis with h = w = 0 (the reference's convention for
    non-video rows, h3_inference/tests/tempo.py:98-111)."""
    t, h, w = grid_thw
    tt = torch.arange(t, device=device).repeat_interleave(h * w)
    hh = torch.arange(h, device=device).repeat_interleave(w).repeat(t)
    ww = torch.arange(w, device=device).repeat(t * h)
    video = torch.stack([tt, hh, ww], dim=1)
    audio = torch.zeros(audio_tokens, 3, dtype=video.dtype, device=device)
    audio[:, 0] = torch.arange(audio_tokens, device=device)
    return torch.cat([video, audio], dim=0).to(torch.float32)
