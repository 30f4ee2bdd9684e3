"""DiT sub-blocks on the NVFP4 kernels.

``FFNBlock`` is the feed-forward half of a DiT block in the GELU/bias
configuration: RMSNorm (optionally adaLN-modulated) -> NVFP4 up-projection
(+b1, GELU-tanh, |u| max in the epilogue) -> NVFP4 re-quantization of u ->
NVFP4 down-projection (+b2) + residual.  It is what the reference reaches
through ``norm_modulate`` + ``ffn`` + ``gate_residual``
(h3_inference/transformer/model.py:200-207,
h3_inference/kernels/ffn_qkvo_gemms.py:45-54) with the GEMMs on
``torch._scaled_mm`` and the elementwise work on torch.compile.

Launches per call: RMSNorm stats, RMSNorm->NVFP4, GEMM-up, quantize,
GEMM-down (5 kernels) plus one 4-byte memset.  All intermediates live in a
per-(T, device) workspace that is allocated once.
"""
from __future__ import annotations

import torch

from . import ops
from .nvfp4 import NVFP4Weight


class FFNBlock:
    def __init__(self, w1: torch.Tensor, b1: torch.Tensor | None, w2: torch.Tensor,
                 b2: torch.Tensor | None, gamma: torch.Tensor, eps: float = 1e-6):
        self.w1 = NVFP4Weight(w1)
        self.w2 = NVFP4Weight(w2)
        self.b1 = None if b1 is None else b1.to(torch.bfloat16).contiguous()
        self.b2 = None if b2 is None else b2.to(torch.bfloat16).contiguous()
        self.gamma = gamma.to(torch.bfloat16).contiguous()
        self.eps = float(eps)
        self.hidden = self.w1.in_features
        self.ffn_dim = self.w1.out_features
        self._ws: dict[tuple, dict] = {}
        # When a list, (start, end) CUDA events are appended around every GEMM
        # launch on the current stream (used to time the dominant kernel).
        self.gemm_events: list | None = None

    def flops(self, tokens: int) -> int:
        return 2 * tokens * self.hidden * self.ffn_dim * 2

    def _workspace(self, T: int, dev: torch.device) -> dict:
        key = (T, dev)
        ws = self._ws.get(key)
        if ws is None:
            Tp = ops.pad_m(T)
            F = self.ffn_dim
            ws = {
                "norm": {},
                "u": torch.empty(T, F, dtype=torch.bfloat16, device=dev),
                "amax_u": torch.zeros(1, dtype=torch.float32, device=dev),
                "qu": torch.empty(Tp, F // 2, dtype=torch.uint8, device=dev),
                "sfu": torch.empty(Tp * (F // 16), dtype=torch.uint8, device=dev),
                "gsu": torch.empty(1, dtype=torch.float32, device=dev),
            }
            self._ws[key] = ws
        return ws

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None, *,
                 shift: torch.Tensor | None = None, scale: torch.Tensor | None = None,
                 mod_idx: torch.Tensor | None = None) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        T = x2.shape[0]
        ws = self._workspace(T, x.device)
        qh, sfh, gsh = ops.rmsnorm_quantize(x2, self.gamma, self.eps, shift=shift, scale=scale,
                                            mod_idx=mod_idx, ws=ws["norm"])
        ws["amax_u"].zero_()
        ev = self._event()
        u = ops.gemm(qh, sfh, gsh, T, self.w1.qdata, self.w1.scale_u8, self.w1.global_scale,
                     self.ffn_dim, self.hidden, bias=self.b1, act=ops.ACT_GELU_TANH,
                     out=ws["u"], amax_out=ws["amax_u"])
        self._event(ev)
        qu, sfu, gsu = ops.quantize(u, mpad=qh.shape[0], amax_t=ws["amax_u"], q_out=ws["qu"],
                                    sf_out=ws["sfu"], gs_out=ws["gsu"])
        ev = self._event()
        y = ops.gemm(qu, sfu, gsu, T, self.w2.qdata, self.w2.scale_u8, self.w2.global_scale,
                     self.hidden, self.ffn_dim, bias=self.b2, residual=x2, out=out)
        self._event(ev)
        return y.reshape(shape)

    def _event(self, start=None):
        if self.gemm_events is None:
            return None
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        if start is not None:
            self.gemm_events.append((start, e))
        return e
