"""The KATA mixer around the attention op, on this library's kernels.

``kata/layer.py`` (``KataAttention.forward`` :286-541, the ``FlashKata`` path) runs, per layer:
q/k/v projections, a causal short convolution with SiLU on each (fla ``ShortConvolution``), the
optional qk normalisation (l2 or RMSNorm) and RoPE, the KATA-SPD attention op, a per-head output
RMSNorm over ``head_v_dim`` and the output projection.  Here the same steps run as:

* one GEMM for the three projections (the weights stay three parameters with the reference's
  names, concatenated per call), then ``kata_short_conv_fwd`` reading q, k and v as column ranges
  of that output and writing them contiguous, ready for the attention kernels' tensor maps (its
  backward writes the three input gradients into one buffer, so the projection backward is again
  one GEMM);
* ``kata_rownorm_fwd`` for the qk normalisation fused with RoPE (one pass per tensor);
* the attention autograd ops of :mod:`linatt_b200.parallel_kata_attn`;
* ``kata_rownorm_fwd`` for the output RMSNorm.

Every step has its backward on the GPU (``kata_short_conv_bwd``, ``kata_rownorm_bwd``); the weight
gradients of the convolution and the norms come out in fp32.  There is no CPU path.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib
from .parallel_kata_attn import parallel_kata_attn, parallel_kata_attn_decay, parallel_kata_attn_sum

__all__ = ["short_conv", "ShortConvQKVFunction", "row_norm", "RowNormFunction", "rope_tables", "FlashKataMixer"]


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _lib.DTYPE[t.dtype]
    except KeyError as e:
        raise TypeError(f"unsupported dtype {t.dtype}") from e


def _rows_view(x: torch.Tensor) -> tuple[int, int]:
    """(B, T) and row stride (elements) of a (B, T, C) tensor whose last dim is contiguous."""
    if x.dim() != 3 or x.stride(-1) != 1 or x.stride(0) != x.shape[1] * x.stride(1):
        raise ValueError("expected a (B, T, C) tensor with contiguous channels and rows")
    return x.stride(1)


class ShortConvQKVFunction(torch.autograd.Function):
    """Causal depthwise convolution (+ SiLU) of several column ranges of one (B, T, Ctot) tensor.

    ``forward(ctx, x, activation, *weights)``: ``x`` is the fused projection output; the weights
    are (C_i, 1, K) fp32 tensors (``nn.Conv1d`` layout) whose C_i add up to Ctot.  Returns one
    contiguous (B, T, C_i) tensor per weight.  Backward returns dx as one (B, T, Ctot) tensor and
    each weight's gradient in fp32.  Reference semantics: fla ``ShortConvolution`` (causal padding
    K - 1, no bias in the layer's configs, ``activation="silu"``)."""

    @staticmethod
    def forward(ctx, x, activation, *weights):
        dev = _lib.require_cuda(x, *weights)
        B, T, Ctot = x.shape
        ldx = _rows_view(x)
        if sum(w.shape[0] for w in weights) != Ctot:
            raise ValueError("the convolution widths must add up to the channel count of x")
        outs = []
        off = 0
        L = _lib.lib()
        st = _lib.stream_handle(dev)
        for w in weights:
            C, _, K = w.shape
            y = torch.empty(B, T, C, device=dev, dtype=x.dtype)
            wf = w.detach().reshape(C, K).float().contiguous()
            a = _lib.ConvArgs(x=x.data_ptr() + off * x.element_size(), w=wf.data_ptr(), bias=None, y=y.data_ptr(),
                              dtype=_dtype_code(x), B=B, T=T, C=C, K=K, ldx=ldx, ldy=C, lddx=C,
                              activation=int(activation))
            _lib.check(L.kata_short_conv_fwd(ctypes_ref(a), st), "kata_short_conv_fwd")
            outs.append(y)
            off += C
        ctx.save_for_backward(x, *weights)
        ctx.activation = int(activation)
        return tuple(outs)

    @staticmethod
    def backward(ctx, *grads):
        x, *weights = ctx.saved_tensors
        dev = x.device
        B, T, Ctot = x.shape
        ldx = _rows_view(x)
        dx = torch.empty(B, T, Ctot, device=dev, dtype=x.dtype)
        L = _lib.lib()
        st = _lib.stream_handle(dev)
        dws = []
        off = 0
        for w, g in zip(weights, grads):
            C, _, K = w.shape
            g = torch.zeros(B, T, C, device=dev, dtype=x.dtype) if g is None else g.to(x.dtype).contiguous()
            wf = w.detach().reshape(C, K).float().contiguous()
            dw = torch.empty(C, K, device=dev, dtype=torch.float32)
            a = _lib.ConvArgs(x=x.data_ptr() + off * x.element_size(), w=wf.data_ptr(), bias=None, dy=g.data_ptr(),
                              dx=dx.data_ptr() + off * dx.element_size(), dw=dw.data_ptr(), dtype=_dtype_code(x),
                              B=B, T=T, C=C, K=K, ldx=ldx, ldy=C, lddx=Ctot, activation=ctx.activation)
            nb = L.kata_short_conv_bwd_workspace_bytes(ctypes_ref(a))
            ws = torch.empty(max(nb, 16), device=dev, dtype=torch.uint8)
            a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
            _lib.check(L.kata_short_conv_bwd(ctypes_ref(a), st), "kata_short_conv_bwd")
            dws.append(dw.view(C, 1, K).to(w.dtype))
            off += C
        return (dx, None, *dws)


def ctypes_ref(a):
    import ctypes

    return ctypes.byref(a)


def short_conv(x: torch.Tensor, weight: torch.Tensor, activation: bool = True) -> torch.Tensor:
    """Causal depthwise short convolution (+ SiLU) of a (B, T, C) tensor with an (C, 1, K) weight."""
    return ShortConvQKVFunction.apply(x, activation, weight)[0]


class RowNormFunction(torch.autograd.Function):
    """Row normalisation (l2 / RMS, optional fp32 weight) with optional RoPE, on (rows, N) rows.

    ``norm``: 0 none, 1 l2, 2 RMS; ``rope``: 0 none, 1 interleaved over the row, 2 half-rotation
    in groups of ``R``; ``cos``/``sin``: (T, R/2) fp32 tables; row r is position (r / heads) % T."""

    @staticmethod
    def forward(ctx, x, weight, cos, sin, norm, rope, R, eps, heads, T):
        dev = _lib.require_cuda(x, weight, cos, sin)
        xs = x.contiguous()
        N = xs.shape[-1]
        rows = xs.numel() // N if N else 0
        y = torch.empty_like(xs)
        rstd = torch.empty(rows, device=dev, dtype=torch.float32) if norm else None
        wf = None if weight is None else weight.detach().float().contiguous()
        a = _lib.RowNormArgs(x=xs.data_ptr(), w=_lib.ptr(wf), cos=_lib.ptr(cos), sin=_lib.ptr(sin), y=y.data_ptr(),
                             rstd=_lib.ptr(rstd), dtype=_dtype_code(xs), rows=rows, N=N, T=int(T), heads=int(heads),
                             norm=int(norm), rope=int(rope), R=int(R), eps=float(eps))
        _lib.check(_lib.lib().kata_rownorm_fwd(ctypes_ref(a), _lib.stream_handle(dev)), "kata_rownorm_fwd")
        ctx.save_for_backward(xs, wf, cos, sin, rstd)
        ctx.cfg = (norm, rope, R, eps, heads, T, weight is not None, None if weight is None else weight.dtype)
        return y

    @staticmethod
    def backward(ctx, dy):
        xs, wf, cos, sin, rstd = ctx.saved_tensors
        norm, rope, R, eps, heads, T, has_w, wdt = ctx.cfg
        dev = xs.device
        N = xs.shape[-1]
        rows = xs.numel() // N if N else 0
        dy = dy.to(xs.dtype).contiguous()
        dx = torch.empty_like(xs)
        want_dw = has_w and norm == 2 and ctx.needs_input_grad[1]
        dw = torch.empty(N, device=dev, dtype=torch.float32) if want_dw else None
        a = _lib.RowNormArgs(x=xs.data_ptr(), w=_lib.ptr(wf), cos=_lib.ptr(cos), sin=_lib.ptr(sin), rstd=_lib.ptr(rstd),
                             dy=dy.data_ptr(), dx=dx.data_ptr(), dw=_lib.ptr(dw), dtype=_dtype_code(xs), rows=rows,
                             N=N, T=int(T), heads=int(heads), norm=int(norm), rope=int(rope), R=int(R),
                             eps=float(eps))
        L = _lib.lib()
        nb = L.kata_rownorm_bwd_workspace_bytes(ctypes_ref(a))
        ws = torch.empty(max(nb, 16), device=dev, dtype=torch.uint8)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        _lib.check(L.kata_rownorm_bwd(ctypes_ref(a), _lib.stream_handle(dev)), "kata_rownorm_bwd")
        return dx, (dw.to(wdt) if want_dw else None), None, None, None, None, None, None, None, None


def row_norm(x, weight=None, *, norm="rms", eps=1e-5, cos=None, sin=None, rope=0, rope_dim=0, heads=1, T=1):
    """Normalise the last dimension of ``x`` ("l2", "rms" or None) and optionally rotate it."""
    code = {None: 0, "none": 0, "l2": 1, "rms": 2, "rmsnorm": 2}[norm]
    return RowNormFunction.apply(x, weight, cos, sin, code, rope, rope_dim or x.shape[-1], eps, heads, T)


def rope_tables(seqlen: int, dim: int, base: float, device, dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """cos / sin tables (seqlen, dim/2) as fla's RotaryEmbedding builds them (fp32 angles, rounded
    to the activations' dtype), returned in fp32 for the kernels."""
    inv_freq = 1.0 / (base ** (torch.arange(0, dim, 2, device=device, dtype=torch.float32) / dim))
    t = torch.arange(seqlen, device=device, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    return torch.cos(freqs).to(dtype).float().contiguous(), torch.sin(freqs).to(dtype).float().contiguous()


class FlashKataMixer(nn.Module):
    """``FlashKata`` / ``KataAttention`` (kata/layer.py:45-292 constructor, :286-541 forward) with
    the quadratic feature maps, on this library's kernels.  Same constructor arguments and parameter
    names (``q_proj``, ``k_proj``, ``v_proj``, ``{q,k,v}_conv1d``, ``q_norm``, ``k_norm``, ``norm``,
    ``o_proj``, ``a_proj``, ``dt_proj``, ``A_log``, ``dt_bias``), so a reference state dict loads as is.
    ``forward(hidden_states)`` returns ``(o, None, None)`` like the reference.  Caches
    (``past_key_values``) are not supported: generation uses :mod:`linatt_b200.kata_decode`."""

    def __init__(self, mode: str = "chunk", hidden_size: int = 1024, expand_k: float = 1.0, expand_v: float = 1.0,
                 num_heads: int = 8, num_kv_heads: int | None = None, feature_map: str = "kata_quadratic",
                 spd_num_groups: int = 1, use_offset_gate: bool = False, use_decay: bool = False,
                 qk_norm: bool = False, norm_q="rmsnorm", norm_k="rmsnorm", use_short_conv: bool = False,
                 conv_size: int = 4, conv_bias: bool = False, output_norm: str = "rmsnorm",
                 elementwise_affine: bool = True, norm_eps: float = 1e-5, use_rope: bool = False,
                 rope_theta: float = 10000.0, rope_group: bool = False, max_position_embeddings: int = 2048,
                 layer_idx: int | None = None, **kwargs):
        super().__init__()
        if feature_map not in ("kata_quadratic", "kata_quadratic_sum"):
            raise ValueError("FlashKataMixer requires feature_map in {kata_quadratic, kata_quadratic_sum}")
        if conv_bias:
            raise ValueError("conv_bias=True is not supported (the reference configs use conv_bias=False)")
        self.hidden_size = hidden_size
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads if num_kv_heads is not None else num_heads
        self.num_kv_groups = num_heads // self.num_kv_heads
        self.key_dim = int(hidden_size * expand_k)
        self.value_dim = int(hidden_size * expand_v)
        self.key_dim_per_group = self.key_dim // self.num_kv_groups
        self.value_dim_per_group = self.value_dim // self.num_kv_groups
        self.head_k_dim = self.key_dim // num_heads
        self.head_v_dim = self.value_dim // num_heads
        self.feature_map_name = feature_map
        self.spd_num_groups = spd_num_groups
        self.layer_idx = layer_idx
        self.q_proj = nn.Linear(hidden_size, self.key_dim, bias=False)
        self.k_proj = nn.Linear(hidden_size, self.key_dim_per_group, bias=False)
        self.v_proj = nn.Linear(hidden_size, self.value_dim_per_group, bias=False)
        self.use_short_conv = use_short_conv
        self.conv_size = conv_size
        if use_short_conv:
            # nn.Conv1d holds the (C, 1, K) weight exactly as fla's ShortConvolution (a Conv1d
            # subclass) does, with the same initialisation; its own forward is never called.
            mk = lambda c: nn.Conv1d(c, c, conv_size, groups=c, bias=False, padding=conv_size - 1)  # noqa: E731
            self.q_conv1d = mk(self.key_dim)
            self.k_conv1d = mk(self.key_dim_per_group)
            self.v_conv1d = mk(self.value_dim_per_group)
        if isinstance(norm_q, bool):
            norm_q = "rmsnorm"
        if isinstance(norm_k, bool):
            norm_k = "rmsnorm"
        self.qk_norm, self.norm_q, self.norm_k = qk_norm, norm_q, norm_k
        if qk_norm and norm_q == "rmsnorm":
            self.q_norm = _FP32RMSNormWeight(self.head_k_dim)
        if qk_norm and norm_k == "rmsnorm":
            self.k_norm = _FP32RMSNormWeight(self.head_k_dim)
        if output_norm not in ("rmsnorm", "identity"):
            raise ValueError(f"unsupported output_norm {output_norm!r}")
        self.output_norm = output_norm
        if output_norm == "rmsnorm":
            self.norm = _FP32RMSNormWeight(self.head_v_dim, eps=norm_eps, affine=elementwise_affine)
        self.o_proj = nn.Linear(self.value_dim, hidden_size, bias=False)
        self.use_rope, self.rope_group, self.rope_theta = use_rope, rope_group, rope_theta
        self.max_position_embeddings = max_position_embeddings
        self.use_offset_gate = use_offset_gate
        if use_offset_gate:
            if self.num_kv_groups != 1:
                raise ValueError("use_offset_gate currently requires MHA (num_kv_heads=num_heads)")
            self._off_E = self.head_k_dim // spd_num_groups
            self._off_Epad = max(16, 1 << self._off_E.bit_length())
            self._off_scale = 1.0 / math.sqrt(self._off_E)
            self.a_proj = nn.Linear(hidden_size, num_heads, bias=True)
        self.use_decay = use_decay
        if use_decay:
            if feature_map != "kata_quadratic":
                raise ValueError("use_decay currently requires feature_map=kata_quadratic (concat)")
            self.dt_proj = nn.Linear(hidden_size, num_heads, bias=False)
            A = torch.empty(num_heads).uniform_(0, 16)
            self.A_log = nn.Parameter(torch.log(A))
            dt = torch.exp(torch.rand(num_heads) * (math.log(0.1) - math.log(0.001)) + math.log(0.001)).clamp(min=1e-4)
            self.dt_bias = nn.Parameter(dt + torch.log(-torch.expm1(-dt)))

    # -- helpers -------------------------------------------------------------------------------
    def _augment_offset(self, q, k, off):
        # Same packing as kata/layer.py:268-282 (append the gate to each q group, 1 to each k group,
        # zero-pad each group to a power of two).
        B, T, H, _ = q.shape
        M, E, Ep = self.spd_num_groups, self._off_E, self._off_Epad

        def _pack(x, col):
            xg = x.view(B, T, x.shape[2], M, E)
            c = col[..., None, None].expand(B, T, x.shape[2], M, 1).to(x.dtype)
            z = x.new_zeros(B, T, x.shape[2], M, Ep - E - 1)
            return torch.cat([xg, c, z], dim=-1).reshape(B, T, x.shape[2], M * Ep)

        return _pack(q, off), _pack(k, torch.ones_like(off))

    def _qk_prologue(self, x, norm_kind, weight, T, cos, sin):
        """qk normalisation then RoPE on a (B, T, H, D) tensor, one pass."""
        norm = {False: 0, "l2": 1, "rmsnorm": 2}[norm_kind if self.qk_norm else False]
        rope = 0 if not self.use_rope else (2 if self.rope_group else 1)
        if norm == 0 and rope == 0:
            return x
        R = (self.head_k_dim // self.spd_num_groups) if self.rope_group else self.head_k_dim
        B, T_, H, D = x.shape
        eps = 1e-6 if norm == 1 else (weight.eps if weight is not None else 1e-5)
        y = RowNormFunction.apply(x.reshape(B * T_ * H, D), None if weight is None else weight.weight, cos, sin, norm,
                                  rope, R, eps, H, T_)
        return y.view(B, T_, H, D)

    def forward(self, hidden_states: torch.Tensor, attention_mask: torch.Tensor | None = None,
                past_key_values=None, use_cache: bool | None = False, **kwargs):
        if past_key_values is not None or use_cache:
            raise NotImplementedError("FlashKataMixer keeps no cache; use linatt_b200.kata_decode for generation")
        B, T, _ = hidden_states.shape
        w = torch.cat([self.q_proj.weight, self.k_proj.weight, self.v_proj.weight], dim=0)
        qkv = F.linear(hidden_states, w)  # one GEMM for the three projections
        Cq, Ck = self.key_dim, self.key_dim_per_group
        if self.use_short_conv:
            q, k, v = ShortConvQKVFunction.apply(qkv, True, self.q_conv1d.weight, self.k_conv1d.weight,
                                                 self.v_conv1d.weight)
        else:
            q, k, v = qkv[..., :Cq], qkv[..., Cq:Cq + Ck], qkv[..., Cq + Ck:]
        if attention_mask is not None:
            v = v.mul(attention_mask[:, -v.shape[-2]:, None])
        q = q.reshape(B, T, self.num_heads, self.head_k_dim)
        k = k.reshape(B, T, self.num_kv_heads, self.head_k_dim)
        v = v.reshape(B, T, self.num_kv_heads, self.head_v_dim)
        cos = sin = None
        if self.use_rope:
            dim = (self.head_k_dim // self.spd_num_groups) if self.rope_group else self.head_k_dim
            cos, sin = rope_tables(max(T, self.max_position_embeddings), dim, self.rope_theta, q.device, q.dtype)
        q = self._qk_prologue(q, self.norm_q, getattr(self, "q_norm", None), T, cos, sin)
        k = self._qk_prologue(k, self.norm_k, getattr(self, "k_norm", None), T, cos, sin)
        is_sum = self.feature_map_name == "kata_quadratic_sum"
        q_in, k_in, scale_in = q, k, None
        if self.use_offset_gate:
            off = torch.sigmoid(self.a_proj(hidden_states))
            q_in, k_in = self._augment_offset(q, k, off)
            scale_in = self._off_scale
        if self.use_decay:
            dt = F.softplus(self.dt_proj(hidden_states) + self.dt_bias)
            c = (-self.A_log.float().exp() * dt.float()).cumsum(dim=1).contiguous()
            o = parallel_kata_attn_decay(q_in, k_in, v, c, num_groups=self.spd_num_groups, scale=scale_in)
        elif is_sum:
            o = parallel_kata_attn_sum(q_in, k_in, v, num_groups=self.spd_num_groups, scale=scale_in)
        else:
            o = parallel_kata_attn(q_in, k_in, v, num_groups=self.spd_num_groups, scale=scale_in)
        if self.output_norm == "rmsnorm":
            Hq, Dv = o.shape[2], o.shape[3]
            o = RowNormFunction.apply(o.reshape(B * T * Hq, Dv), self.norm.weight, None, None, 2, 0, Dv,
                                      self.norm.eps, Hq, T).view(B, T, Hq, Dv)
        o = self.o_proj(o.reshape(B, T, -1))
        return o, None, past_key_values


class _FP32RMSNormWeight(nn.Module):
    """Holds an fp32 RMSNorm scale under the name ``weight`` (fla ``RMSNorm(dim, dtype=float32)``);
    the normalisation itself runs in ``kata_rownorm_*``."""

    def __init__(self, dim: int, eps: float = 1e-5, affine: bool = True):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim, dtype=torch.float32)) if affine else None
