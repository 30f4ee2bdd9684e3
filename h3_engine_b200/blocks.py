"""DiT sub-blocks on the sm_100a kernels.

``FFNBlock`` -- the feed-forward half of a DiT block (GELU/bias
configuration): RMSNorm (optionally adaLN-modulated) -> NVFP4 up-projection
(+b1, GELU-tanh, |u| max in the epilogue) -> NVFP4 re-quantization of u ->
NVFP4 down-projection (+b2, optional adaLN gate) + residual.  The reference
reaches this through ``norm_modulate`` + ``ffn`` + ``gate_residual``
(h3_inference/transformer/model.py:200-207,
h3_inference/kernels/ffn_qkvo_gemms.py:45-54).

``AttnBlock`` -- the attention half: RMSNorm (+modulation) -> NVFP4 QKV
projection (one GEMM; q/k/v weights keep their own global scales) -> per-head
qk RMSNorm + 3D RoPE in place -> packed varlen attention -> NVFP4
quantization of the attention output -> NVFP4 out-projection (+gate) +
residual (h3_inference/transformer/model.py:81-106,191-198).  With a
``SequenceShard`` the block runs on this rank's token rows: the projection
writes Q locally and K|V straight into this rank's rows of the full-sequence
K|V buffer, one in-place NCCL all-gather completes it, and attention reads
local queries against all keys.

``DiTBlock`` -- attention then FFN with the six adaLN-zero tables (shift /
scale / gate per half), gathered per token by ``mod_idx``.

All intermediates live in per-(rows, device) workspaces allocated once.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops
from .nvfp4 import NVFP4Weight


_GEMM_SINK = object()


class _GemmTimer:
    """When ``gemm_events`` / ``attn_events`` are lists, (start, end) CUDA
    events are appended around every GEMM / attention launch on the current
    stream (how bench.py times the dominant kernels inside a real step)."""

    gemm_events: list | None = None
    attn_events: list | None = None

    def _event(self, start=None, sink=_GEMM_SINK):
        """Record an event; with ``start`` append (start, event) to ``sink``
        (default the GEMM list; a None sink records nothing)."""
        if sink is _GEMM_SINK:
            sink = self.gemm_events
        if sink is None:
            return None
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        if start is not None:
            sink.append((start, e))
        return e


def _buf(ws: dict, name: str, shape, dtype, dev) -> torch.Tensor:
    t = ws.get(name)
    if t is None or t.shape != torch.Size(shape) or t.dtype != dtype:
        t = torch.empty(shape, dtype=dtype, device=dev)
        ws[name] = t
    return t


class FFNBlock(_GemmTimer):
    """FFN half of a DiT block: RMSNorm (+adaLN modulation) -> NVFP4 -> up
    GEMM with the activation in its epilogue -> re-quantization -> down GEMM
    (+bias, adaLN gate, residual).  ``act="gelu"``: GELU-tanh with bias (the
    configuration of this model); ``act="swiglu"``: the reference model's
    SwiGLU feed-forward (``w1`` the fused [value | gate] projection, 2F rows,
    no bias; h3_inference/transformer/ops.py:62-81)."""

    def __init__(self, w1: torch.Tensor, b1: torch.Tensor | None, w2: torch.Tensor,
                 b2: torch.Tensor | None, gamma: torch.Tensor, eps: float = 1e-6,
                 workspace: dict | None = None, act: str = "gelu"):
        if act not in ("gelu", "swiglu"):
            raise ValueError(f"unknown FFN activation {act!r}")
        self.act = act
        if act == "swiglu":
            if b1 is not None:
                raise ValueError("the SwiGLU feed-forward carries no up-projection bias")
            if w1.shape[0] % 256:
                raise ValueError("SwiGLU up-projection rows (2F) must be a multiple of 256")
            w1 = w1[ops.swiglu_rows(w1.shape[0] // 2).to(w1.device)]
        self.w1 = NVFP4Weight(w1)
        self.w2 = NVFP4Weight(w2)
        self.b1 = None if b1 is None else b1.to(torch.bfloat16).contiguous()
        self.b2 = None if b2 is None else b2.to(torch.bfloat16).contiguous()
        self.gamma = gamma.to(torch.bfloat16).contiguous()
        self.eps = float(eps)
        self.hidden = self.w1.in_features
        self.ffn_dim = self.w1.out_features // (2 if act == "swiglu" else 1)
        # blocks that run one after another on one stream may share one pool
        self._ws: dict[tuple, dict] = {} if workspace is None else workspace
        self.gemm_events = None

    def flops(self, tokens: int) -> int:
        return 2 * tokens * self.hidden * (self.w1.out_features + self.ffn_dim)

    def _workspace(self, T: int, dev: torch.device) -> dict:
        key = ("ffn", T, self.hidden, self.ffn_dim, dev)
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
                 gate: torch.Tensor | None = None, mod_idx: torch.Tensor | None = None,
                 shard: "SequenceShard | None" = None) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        T = x2.shape[0]
        ws = self._workspace(T, x.device)
        hook = None if shard is None else shard.reduce_max
        qh, sfh, gsh = ops.rmsnorm_quantize(x2, self.gamma, self.eps, shift=shift, scale=scale,
                                            mod_idx=mod_idx, ws=ws["norm"], amax_hook=hook)
        ws["amax_u"].zero_()
        ev = self._event()
        act = ops.ACT_SWIGLU if self.act == "swiglu" else ops.ACT_GELU_TANH
        u = ops.gemm(qh, sfh, gsh, T, self.w1.qdata, self.w1.scale_u8, self.w1.global_scale,
                     self.w1.out_features, self.hidden, bias=self.b1, act=act,
                     out=ws["u"], amax_out=ws["amax_u"])
        self._event(ev)
        if hook is not None:
            hook(ws["amax_u"])
        qu, sfu, gsu = ops.quantize(u, mpad=qh.shape[0], amax_t=ws["amax_u"], q_out=ws["qu"],
                                    sf_out=ws["sfu"], gs_out=ws["gsu"])
        ev = self._event()
        y = ops.gemm(qu, sfu, gsu, T, self.w2.qdata, self.w2.scale_u8, self.w2.global_scale,
                     self.hidden, self.ffn_dim, bias=self.b2, residual=x2, gate=gate,
                     gate_idx=mod_idx if gate is not None else None, out=out)
        self._event(ev)
        return y.reshape(shape)


@dataclass
class SequenceShard:
    """This rank's slice ``[row0, row0 + rows)`` of a token-sharded sequence of
    ``total`` rows, and its collectives:

    * ``all_gather(full, local)``: complete the ``[total, C]`` K|V buffer whose
      rows ``[row0, row0 + rows)`` (``local``) this rank wrote; None when the
      sequence is not split (rows == total, e.g. a CFG-split run);
    * ``reduce_max(t)``: in-place max over every rank holding part of the
      activation tensor of a 1-element fp32 amax, so every NVFP4 quantization
      uses the global scale of the whole tensor (the distributed run then
      computes the same bytes as the single-GPU one).
    """

    row0: int
    rows: int
    total: int
    all_gather: object
    reduce_max: object = None
    chunk: int = 0        # rows per shard in the gathered buffer (0: ``rows``)
    parts: int = 0        # shards (0: ceil(total / chunk))

    def buffer_rows(self) -> int:
        chunk = self.chunk or self.rows
        parts = self.parts or -(-self.total // chunk)
        return max(self.total, chunk * parts)


class AttnBlock(_GemmTimer):
    def __init__(self, wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor, wo: torch.Tensor,
                 gamma: torch.Tensor, norm_q: torch.Tensor | None, norm_k: torch.Tensor | None,
                 heads: int, eps: float = 1e-6, qk_eps: float = 1e-6,
                 bo: torch.Tensor | None = None, workspace: dict | None = None):
        ws = [NVFP4Weight(w) for w in (wq, wk, wv)]
        self.heads = heads
        self.inner = ws[0].out_features
        self.head_dim = self.inner // heads
        self.hidden = ws[0].in_features
        # q|k|v packed weights concatenated along N, one global scale each
        self.w_qkv = torch.cat([w.qdata for w in ws]).contiguous()
        self.sf_qkv = torch.cat([w.scale_u8 for w in ws]).contiguous()
        self.gs_qkv = torch.cat([w.global_scale for w in ws]).contiguous()
        self.wo = NVFP4Weight(wo)
        self.bo = None if bo is None else bo.to(torch.bfloat16).contiguous()
        self.gamma = gamma.to(torch.bfloat16).contiguous()
        self.norm_q = None if norm_q is None else norm_q.to(torch.bfloat16).contiguous()
        self.norm_k = None if norm_k is None else norm_k.to(torch.bfloat16).contiguous()
        self.eps, self.qk_eps = float(eps), float(qk_eps)
        self._ws: dict[tuple, dict] = {} if workspace is None else workspace
        self.gemm_events = None

    def flops(self, tokens: int, cu_seqlens) -> dict:
        hd, d = self.inner, self.hidden
        cu = list(cu_seqlens)
        attn = sum(4 * hd * (b - a) ** 2 for a, b in zip(cu[:-1], cu[1:]))
        return {"nvfp4": 2 * tokens * d * 3 * hd + 2 * tokens * hd * d, "attention": attn}

    def _sf_rows(self, r0: int, r1: int) -> torch.Tensor:
        per_row = self.hidden // 16           # scale bytes per weight row (blocked layout)
        return self.sf_qkv[r0 * per_row:r1 * per_row]

    # K|V of a token-sharded block is projected, normed and all-gathered in
    # this many head groups, each group's gather running on the side stream
    # under the next group's projection and the previous group's attention
    kv_groups = 2

    def _kv_group_weights(self, G: int) -> list:
        """Per head group g: the packed weight rows [K heads of g | V heads of
        g] (2 * HD / G rows), their blocked scales (whole 128-row tiles, so a
        row range is a contiguous byte range) and their global scales
        [gs_k, gs_v], one per HD / G output columns.  Built once per G."""
        cache = self.__dict__.setdefault("_kvg", {})
        if G in cache:
            return cache[G]
        HD, per_row = self.inner, self.hidden // 16
        hg = HD // G
        groups = []
        for g in range(G):
            k0, v0 = HD + g * hg, 2 * HD + g * hg
            w = torch.cat([self.w_qkv[k0:k0 + hg], self.w_qkv[v0:v0 + hg]]).contiguous()
            sf = torch.cat([self.sf_qkv[k0 * per_row:(k0 + hg) * per_row],
                            self.sf_qkv[v0 * per_row:(v0 + hg) * per_row]]).contiguous()
            groups.append((w, sf, self.gs_qkv[1:3].contiguous()))
        cache[G] = groups
        return groups

    def _groups_for(self, shard) -> int:
        G = self.kv_groups
        while G > 1 and (self.heads % G or (self.inner // G) % 128):
            G -= 1
        return G

    def _sharded_attention(self, qh, sfh, gsh, T, ws, dev, cos, sin, cu_seqlens, shard):
        """Token-sharded attention: for each head group, this rank's K|V rows
        (projection + key norm/RoPE) go into its chunk of that group's
        full-sequence buffer and are all-gathered on a side stream while the
        main stream moves on (the next group's projection, the query
        projection and norm/RoPE, then attention group by group, each waiting
        only for its own gather).  Every byte equals the unsharded run's (GEMM
        columns do not depend on the N split; heads are independent)."""
        HD, H, D = self.inner, self.heads, self.head_dim
        G = self._groups_for(shard)
        hg, Hg = HD // G, H // G
        groups = self._kv_group_weights(G)
        q = _buf(ws, "q", (T, HD), torch.bfloat16, dev)
        kvs = [_buf(ws, f"kv{g}", (shard.buffer_rows(), 2 * hg), torch.bfloat16, dev)
               for g in range(G)]
        main = torch.cuda.current_stream(dev)
        side = ws.get("side")
        if side is None:
            side = ws["side"] = torch.cuda.Stream(device=dev)
        gathered = []
        ev = self._event()
        for g, (w, sf, gs) in enumerate(groups):
            kv_local = kvs[g][shard.row0:shard.row0 + T]
            ops.gemm(qh, sfh, gsh, T, w, sf, gs, 2 * hg, self.hidden, gsb_seg=hg, out=kv_local)
            ops.qk_norm_rope(kv_local, Hg, D, q_off=0, k_off=0, wq=None, wk=self.norm_k,
                             eps=self.qk_eps, cos=cos, sin=sin, heads_q=False)
            ready = torch.cuda.Event()
            ready.record(main)
            side.wait_event(ready)
            with torch.cuda.stream(side):
                shard.all_gather(kvs[g], kv_local)
                done = torch.cuda.Event()
                done.record(side)
            gathered.append(done)
        ops.gemm(qh, sfh, gsh, T, self.w_qkv[:HD], self._sf_rows(0, HD), self.gs_qkv[:1], HD,
                 self.hidden, out=q)
        ops.qk_norm_rope(q, H, D, q_off=0, k_off=0, wq=self.norm_q, wk=None, eps=self.qk_eps,
                         cos=cos, sin=sin, heads_k=False)
        self._event(ev)
        o = _buf(ws, "o", (T, HD), torch.bfloat16, dev)
        for g in range(G):
            # also orders the next block's writes to this group's buffer after the gather
            main.wait_event(gathered[g])
            ev = self._event(sink=self.attn_events)
            ops.attention_varlen(q, Hg, D, cu_seqlens, q_off=g * hg, k_off=0, v_off=hg,
                                 kv=kvs[g][:shard.total], q_row0=shard.row0,
                                 out=o[:, g * hg:(g + 1) * hg])
            self._event(ev, sink=self.attn_events)
        return o

    def __call__(self, x: torch.Tensor, rope: tuple[torch.Tensor, torch.Tensor] | None,
                 cu_seqlens, out: torch.Tensor | None = None, *,
                 shift: torch.Tensor | None = None, scale: torch.Tensor | None = None,
                 gate: torch.Tensor | None = None, mod_idx: torch.Tensor | None = None,
                 shard: SequenceShard | None = None) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        T = x2.shape[0]
        HD, H, D = self.inner, self.heads, self.head_dim
        dev = x.device
        split = shard is not None and shard.all_gather is not None
        ws = self._ws.setdefault(("attn", T, self.hidden, self.inner, dev, split), {"norm": {}})
        cos, sin = rope if rope is not None else (None, None)
        hook = None if shard is None else shard.reduce_max
        qh, sfh, gsh = ops.rmsnorm_quantize(x2, self.gamma, self.eps, shift=shift, scale=scale,
                                            mod_idx=mod_idx, ws=ws["norm"], amax_hook=hook)
        if shard is None or shard.all_gather is None:
            qkv = _buf(ws, "qkv", (T, 3 * HD), torch.bfloat16, dev)
            ev = self._event()
            ops.gemm(qh, sfh, gsh, T, self.w_qkv, self.sf_qkv, self.gs_qkv, 3 * HD, self.hidden,
                     gsb_seg=HD, out=qkv)
            self._event(ev)
            ops.qk_norm_rope(qkv, H, D, q_off=0, k_off=HD, wq=self.norm_q, wk=self.norm_k,
                             eps=self.qk_eps, cos=cos, sin=sin)
            ev = self._event(sink=self.attn_events)
            o = ops.attention_varlen(qkv, H, D, cu_seqlens, q_off=0, k_off=HD, v_off=2 * HD,
                                     out=_buf(ws, "o", (T, HD), torch.bfloat16, dev))
            self._event(ev, sink=self.attn_events)
        else:
            if shard.rows != T:
                raise ValueError("shard rows do not match the local activation")
            o = self._sharded_attention(qh, sfh, gsh, T, ws, dev, cos, sin, cu_seqlens, shard)
        mp = qh.shape[0]
        amax_o = ops.amax(o, out=_buf(ws, "amax_o", (1,), torch.float32, dev))
        if hook is not None:
            hook(amax_o)
        qo, sfo, gso = ops.quantize(o, mpad=mp, amax_t=amax_o,
                                    q_out=_buf(ws, "qo", (mp, HD // 2), torch.uint8, dev),
                                    sf_out=_buf(ws, "sfo", (mp * (HD // 16),), torch.uint8, dev),
                                    gs_out=_buf(ws, "gso", (1,), torch.float32, dev))
        if out is None:
            out = _buf(ws, "y", (T, self.hidden), torch.bfloat16, dev)
        ev = self._event()
        y = ops.gemm(qo, sfo, gso, T, self.wo.qdata, self.wo.scale_u8, self.wo.global_scale,
                     self.hidden, HD, bias=self.bo, residual=x2, gate=gate,
                     gate_idx=mod_idx if gate is not None else None, out=out)
        self._event(ev)
        return y.reshape(shape)


class DiTBlock:
    """Attention half then FFN half, each ``x + gate * f(modulate(norm(x)))``
    (h3_inference/transformer/model.py:176-209)."""

    def __init__(self, attn: AttnBlock, ffn: FFNBlock):
        self.attn, self.ffn = attn, ffn

    def __call__(self, x: torch.Tensor, rope, cu_seqlens, mod: tuple[torch.Tensor, ...] | None,
                 mod_idx: torch.Tensor | None = None, out: torch.Tensor | None = None,
                 shard: SequenceShard | None = None) -> torch.Tensor:
        if mod is None:
            sa = ca = ga = sm = cm = gm = None
        else:
            sa, ca, ga, sm, cm, gm = mod
        h = self.attn(x, rope, cu_seqlens, shift=sa, scale=ca, gate=ga, mod_idx=mod_idx,
                      shard=shard)
        return self.ffn(h, out=out, shift=sm, scale=cm, gate=gm, mod_idx=mod_idx, shard=shard)
