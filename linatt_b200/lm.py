"""A KATA causal language model whose token mixer is :class:`linatt_b200.mixer.FlashKataMixer`.

Mirrors ``KataForCausalLM`` (kata/modeling.py:33-155) with fla's LinearAttention body: token
embedding, ``num_hidden_layers`` blocks of [RMSNorm -> KATA mixer -> residual -> RMSNorm -> SwiGLU
MLP -> residual], a final RMSNorm and an output head tied to the embedding; the loss is the mean
next-token cross entropy (the last position of every row has no target), as fla's
``LinearAttentionForCausalLM`` computes it.  Parameter names follow the reference
(``model.layers.{i}.attn.*``, ``mlp.gate_proj`` / ``up_proj`` / ``down_proj``, ``attn_norm``,
``mlp_norm``, ``model.norm``, ``lm_head``).  Everything outside the mixer is plain PyTorch
(cuBLAS GEMMs, residual adds, embedding) except the RMSNorms (the mixer's row kernel), the SwiGLU and
the cross entropy (``lm_ops.cu``): the hot path of this library is the mixer.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from .mixer import FlashKataMixer, RowNormFunction

__all__ = ["KataLMConfig", "KataLM"]


@dataclass
class KataLMConfig:
    """Defaults: ``configs/model/200m/kata_quadratic_200m.yaml`` of the reference (the 24-layer,
    d_model 768, 12 x 64 heads, concat score M = 4, short convolution of width 4, vocab 32000 LM)."""

    hidden_size: int = 768
    num_hidden_layers: int = 24
    num_heads: int = 12
    num_kv_heads: int | None = None
    expand_k: float = 1.0
    expand_v: float = 1.0
    feature_map: str = "kata_quadratic"
    spd_num_groups: int = 4
    use_short_conv: bool = True
    conv_size: int = 4
    qk_norm: bool = False
    norm_q: str = "rmsnorm"
    norm_k: str = "rmsnorm"
    use_rope: bool = False
    rope_group: bool = False
    use_offset_gate: bool = False
    use_decay: bool = False
    hidden_ratio: int = 4
    intermediate_size: int | None = None
    max_position_embeddings: int = 2048
    norm_eps: float = 1e-6
    vocab_size: int = 32000
    tie_word_embeddings: bool = True
    initializer_range: float = 0.006
    extra: dict = field(default_factory=dict)

    def mixer_kwargs(self) -> dict:
        return dict(hidden_size=self.hidden_size, expand_k=self.expand_k, expand_v=self.expand_v,
                    num_heads=self.num_heads, num_kv_heads=self.num_kv_heads, feature_map=self.feature_map,
                    spd_num_groups=self.spd_num_groups, use_short_conv=self.use_short_conv,
                    conv_size=self.conv_size, qk_norm=self.qk_norm, norm_q=self.norm_q, norm_k=self.norm_k,
                    use_rope=self.use_rope, rope_group=self.rope_group, use_offset_gate=self.use_offset_gate,
                    use_decay=self.use_decay, norm_eps=self.norm_eps,
                    max_position_embeddings=self.max_position_embeddings, **self.extra)


class RMSNorm(nn.Module):
    """Hidden-state RMSNorm (fla ``RMSNorm``) on ``kata_rownorm_*``: one pass forward, one backward
    pass plus a fixed-order reduction of the fp32 weight gradient."""

    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        N = x.shape[-1]
        return RowNormFunction.apply(x.reshape(-1, N), self.weight, None, None, 2, 0, N, self.eps, 1, 1).view(x.shape)


def _dt(t: torch.Tensor) -> int:
    return _lib.DTYPE[t.dtype]


class AddRMSNormFunction(torch.autograd.Function):
    """(h_out, y) = (h + x, RMSNorm(h + x) * w) on ``kata_add_rmsnorm_*``: the residual add of a block
    output x (bf16 / f16) into the fp32 hidden stream h, fused with the next RMSNorm, whose output is
    produced directly in x's dtype for the following GEMMs.  One pass each way."""

    @staticmethod
    def forward(ctx, h, x, w, eps):
        dev = _lib.require_cuda(h, x, w)
        N = h.shape[-1]
        hc, xc = h.float().contiguous(), x.contiguous()
        rows = hc.numel() // N
        h_out = torch.empty_like(hc)
        y = torch.empty(xc.shape, device=dev, dtype=xc.dtype)
        rstd = torch.empty(rows, device=dev, dtype=torch.float32)
        a = _lib.AddRmsNormArgs(h=hc.data_ptr(), x=xc.data_ptr(), w=w.data_ptr(), h_out=h_out.data_ptr(),
                                y=y.data_ptr(), rstd=rstd.data_ptr(), rows=rows, N=N, dtype=_dt(xc), eps=float(eps))
        _lib.check(_lib.lib().kata_add_rmsnorm_fwd(a, _lib.stream_handle(dev)), "kata_add_rmsnorm_fwd")
        ctx.save_for_backward(h_out, rstd, w)
        ctx.eps, ctx.xdtype = eps, xc.dtype
        return h_out, y

    @staticmethod
    def backward(ctx, dh_out, dy):
        h_out, rstd, w = ctx.saved_tensors
        dev = h_out.device
        N = h_out.shape[-1]
        rows = h_out.numel() // N
        dyc = (dy if dy is not None else torch.zeros(h_out.shape, device=dev)).to(ctx.xdtype).contiguous()
        dinc = dh_out.float().contiguous() if dh_out is not None else None
        dh = torch.empty_like(h_out)
        dx = torch.empty(h_out.shape, device=dev, dtype=ctx.xdtype)
        dw = torch.empty_like(w)
        a = _lib.AddRmsNormArgs(h_out=h_out.data_ptr(), rstd=rstd.data_ptr(), w=w.data_ptr(), dy=dyc.data_ptr(),
                                dh_in=_lib.ptr(dinc), dh=dh.data_ptr(), dx=dx.data_ptr(), dw=dw.data_ptr(),
                                rows=rows, N=N, dtype=_lib.DTYPE[ctx.xdtype], eps=float(ctx.eps))
        L = _lib.lib()
        nb = L.kata_add_rmsnorm_bwd_workspace_bytes(a)
        ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=dev)
        a.workspace, a.workspace_bytes = ws.data_ptr(), nb
        _lib.check(L.kata_add_rmsnorm_bwd(a, _lib.stream_handle(dev)), "kata_add_rmsnorm_bwd")
        return dh, dx, dw, None


def add_rmsnorm(h: torch.Tensor, x: torch.Tensor, norm: "RMSNorm"):
    """(h + x, norm(h + x)) with the sum kept in fp32 and the normalised output in x's dtype (fused
    for 16-bit block outputs and widths that are a multiple of 256; otherwise the add, then ``norm``)."""
    if x.dtype in (torch.bfloat16, torch.float16) and h.shape[-1] % 256 == 0 and h.shape[-1] <= 1024:
        return AddRMSNormFunction.apply(h, x, norm.weight, norm.eps)
    h = h + x
    return h, norm(h)


class SwiGLUFunction(torch.autograd.Function):
    """y = silu(g) * u of a (rows, 2I) tensor [g | u] on ``kata_swiglu_fwd`` / ``_bwd`` (one pass each)."""

    @staticmethod
    def forward(ctx, gu):
        dev = _lib.require_cuda(gu)
        gu = gu.contiguous()
        I = gu.shape[-1] // 2
        y = torch.empty(*gu.shape[:-1], I, device=dev, dtype=gu.dtype)
        rows = gu.numel() // (2 * I)
        _lib.check(_lib.lib().kata_swiglu_fwd(gu.data_ptr(), y.data_ptr(), rows, I, _dt(gu), _lib.stream_handle(dev)),
                   "kata_swiglu_fwd")
        ctx.save_for_backward(gu)
        return y

    @staticmethod
    def backward(ctx, dy):
        (gu,) = ctx.saved_tensors
        dy = dy.to(gu.dtype).contiguous()
        dgu = torch.empty_like(gu)
        I = gu.shape[-1] // 2
        _lib.check(_lib.lib().kata_swiglu_bwd(gu.data_ptr(), dy.data_ptr(), dgu.data_ptr(), gu.numel() // (2 * I), I,
                                              _dt(gu), _lib.stream_handle(gu.device)), "kata_swiglu_bwd")
        return dgu


class CrossEntropyFunction(torch.autograd.Function):
    """Mean cross entropy of (rows, V) logits against int64 targets (negative: ignored), over the
    valid rows, on ``kata_cross_entropy_fwd`` / ``_bwd``: the logits are read once forward and once
    backward in their own dtype (no fp32 copy); the gradient scale comes from device scalars."""

    @staticmethod
    def forward(ctx, logits, targets):
        dev = _lib.require_cuda(logits, targets)
        logits = logits.contiguous()
        targets = targets.contiguous().to(torch.int64)
        rows, V = logits.shape
        lse = torch.empty(rows, device=dev, dtype=torch.float32)
        loss_rows = torch.empty(rows, device=dev, dtype=torch.float32)
        _lib.check(_lib.lib().kata_cross_entropy_fwd(logits.data_ptr(), targets.data_ptr(), lse.data_ptr(),
                                                     loss_rows.data_ptr(), rows, V, _dt(logits),
                                                     _lib.stream_handle(dev)), "kata_cross_entropy_fwd")
        inv = 1.0 / (targets >= 0).sum().clamp_min(1).to(torch.float32)
        ctx.save_for_backward(logits, targets, lse, inv.reshape(1))
        return loss_rows.sum() * inv

    @staticmethod
    def backward(ctx, g):
        logits, targets, lse, inv = ctx.saved_tensors
        rows, V = logits.shape
        dl = torch.empty_like(logits)
        gs = g.detach().to(torch.float32).reshape(1).contiguous()
        _lib.check(_lib.lib().kata_cross_entropy_bwd(logits.data_ptr(), targets.data_ptr(), lse.data_ptr(),
                                                     gs.data_ptr(), inv.data_ptr(), dl.data_ptr(), rows, V,
                                                     _dt(logits), _lib.stream_handle(logits.device)),
                   "kata_cross_entropy_bwd")
        return dl, None


class GatedMLP(nn.Module):
    """SwiGLU MLP (fla ``GatedMLP``): down(silu(gate(x)) * up(x)), intermediate size the multiple of
    256 nearest above 2/3 * hidden_ratio * hidden_size."""

    def __init__(self, hidden_size: int, hidden_ratio: int, intermediate_size: int | None):
        super().__init__()
        if intermediate_size is None:
            intermediate_size = int(hidden_size * hidden_ratio * 2 / 3)
            intermediate_size = 256 * ((intermediate_size + 255) // 256)
        self.gate_proj = nn.Linear(hidden_size, intermediate_size, bias=False)
        self.up_proj = nn.Linear(hidden_size, intermediate_size, bias=False)
        self.down_proj = nn.Linear(intermediate_size, hidden_size, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        gu = F.linear(x, torch.cat([self.gate_proj.weight, self.up_proj.weight], dim=0))  # one GEMM
        return self.down_proj(SwiGLUFunction.apply(gu))


class KataBlock(nn.Module):
    def __init__(self, cfg: KataLMConfig, layer_idx: int):
        super().__init__()
        self.attn_norm = RMSNorm(cfg.hidden_size, cfg.norm_eps)
        self.attn = FlashKataMixer(layer_idx=layer_idx, **cfg.mixer_kwargs())
        self.mlp_norm = RMSNorm(cfg.hidden_size, cfg.norm_eps)
        self.mlp = GatedMLP(cfg.hidden_size, cfg.hidden_ratio, cfg.intermediate_size)

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        h = h + self.attn(self.attn_norm(h))[0]
        return h + self.mlp(self.mlp_norm(h))


class _Body(nn.Module):
    def __init__(self, cfg: KataLMConfig):
        super().__init__()
        self.embeddings = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList(KataBlock(cfg, i) for i in range(cfg.num_hidden_layers))
        self.norm = RMSNorm(cfg.hidden_size, cfg.norm_eps)


class KataLM(nn.Module):
    """``forward(input_ids, labels=None)`` returns the logits, or the loss when labels are given."""

    def __init__(self, cfg: KataLMConfig):
        super().__init__()
        self.config = cfg
        self.model = _Body(cfg)
        self.lm_head = nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False)
        self.apply(self._init)
        if cfg.tie_word_embeddings:
            self.lm_head.weight = self.model.embeddings.weight

    def _init(self, m: nn.Module) -> None:
        if isinstance(m, (nn.Linear, nn.Embedding)):
            nn.init.normal_(m.weight, mean=0.0, std=self.config.initializer_range)

    def forward(self, input_ids: torch.Tensor, labels: torch.Tensor | None = None) -> torch.Tensor:
        h = self.model.embeddings(input_ids)
        layers = self.model.layers
        # the blocks' residual adds fused with the RMSNorm that follows each of them (the next
        # block's or the final norm); the same function as KataBlock.forward applied in turn
        y = layers[0].attn_norm(h)
        for i, blk in enumerate(layers):
            h, y = add_rmsnorm(h, blk.attn(y)[0], blk.mlp_norm)
            nxt = layers[i + 1].attn_norm if i + 1 < len(layers) else self.model.norm
            h, y = add_rmsnorm(h, blk.mlp(y), nxt)
        logits = self.lm_head(y)
        if labels is None:
            return logits
        # next-token targets; the last position of each row has none
        tgt = torch.cat([labels[:, 1:], torch.full_like(labels[:, :1], -100)], dim=1)
        return CrossEntropyFunction.apply(logits.reshape(-1, logits.shape[-1]), tgt.reshape(-1))
