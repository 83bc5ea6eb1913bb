"""Packed-sequence (varlen) form of causal KATA-SPD attention.

Documents are packed along T as (1, T_total, H, D) with ``cu_seqlens`` = [0, l_0, l_0+l_1, ...]
(int, N+1 entries), the layout of the reference's per-document data preparation and of the
``seq_lengths`` / ``seq_starts`` arguments sketched in its unused Hopper kernel
(``kata/kernels/parallel_kata_hopper.py:18-44``).  Token t of document n attends to the tokens
s <= t of document n only.

On the tensor-core kernels (bf16 / f16 inputs in their envelope, with or without decay) the documents go to the
kernels as they lie: each CTA takes one 128-row tile of one document (the tiles of all documents
numbered in document order, ``cu_seqlens`` read on the device), its key tiles start at the
document's first row, and rows past the document's end are masked (their outputs are not written,
and in the backward their per-query vectors are zero).  No padding and no scatter / gather pass.

Otherwise (fp32, shapes outside that envelope) each document is scattered into its own row
of a zero-padded (N, T_max, H, D) batch, the flash kernels run on that batch, and the rows are
gathered back.  Padding sits after each document's last token, so causality keeps it out of every
real row: the outputs and gradients equal those of one call per document.  The cost is the padding
(sum of T_max - l_n tokens) and one scatter / gather pass over q, k, v, o (and their gradients).
"""

from __future__ import annotations

import torch

from . import _lib
from . import parallel_kata_attn as _pka
from .parallel_kata_attn import parallel_kata_attn, parallel_kata_attn_decay, parallel_kata_attn_sum

__all__ = ["varlen_index", "pack_rows", "unpack_rows", "parallel_kata_attn_varlen"]


def varlen_index(cu_seqlens: torch.Tensor, max_seqlen: int | None = None, total: int | None = None):
    """(dst, N, T_max): dst[t] = n * T_max + (t - cu_seqlens[n]) for packed token t of document n.
    ``total`` (= cu_seqlens[-1]) and ``max_seqlen`` spare the device-to-host reads of cu_seqlens."""
    cu = cu_seqlens.to(torch.int64)
    if cu.dim() != 1 or cu.numel() < 2:
        raise ValueError("cu_seqlens must be 1-D with at least two entries")
    lens = cu[1:] - cu[:-1]
    N = lens.numel()
    if max_seqlen is None:
        cpu = cu.cpu()
        if int(cpu[0]) != 0 or bool(((cpu[1:] - cpu[:-1]) < 0).any()):
            raise ValueError("cu_seqlens must start at 0 and be non-decreasing")
        max_seqlen = int((cpu[1:] - cpu[:-1]).max())
    T = int(cu[-1]) if total is None else int(total)
    seq = torch.repeat_interleave(torch.arange(N, device=cu.device), lens, output_size=T)
    pos = torch.arange(seq.numel(), device=cu.device) - cu[seq]
    return seq * max_seqlen + pos, N, max(int(max_seqlen), 1)


def pack_rows(x: torch.Tensor, dst: torch.Tensor, N: int, T_max: int) -> torch.Tensor:
    """(1, T_total, *rest) packed -> (N, T_max, *rest) zero-padded (differentiable)."""
    flat = x[0]
    out = flat.new_zeros((N * T_max,) + tuple(flat.shape[1:]))
    return out.index_copy(0, dst, flat).view((N, T_max) + tuple(flat.shape[1:]))


def unpack_rows(y: torch.Tensor, dst: torch.Tensor) -> torch.Tensor:
    """(N, T_max, *rest) -> (1, T_total, *rest) (differentiable)."""
    return y.reshape((-1,) + tuple(y.shape[2:])).index_select(0, dst).unsqueeze(0)


class _PackedKataFunction(torch.autograd.Function):
    """Packed documents straight through the tensor-core kernels (``cu_seqlens`` on the device);
    ``c`` (1, T_total, HQ) fp32 log-decay or None."""

    @staticmethod
    def forward(ctx, q, k, v, c, cu, num_groups, scale, score):
        o, den = _pka._fwd(q, k, v, num_groups, scale, score, c=c, cu=cu)
        ctx.save_for_backward(q, k, v, o, den, cu, c)
        ctx.num_groups, ctx.scale, ctx.score = num_groups, scale, score
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, den, cu, c = ctx.saved_tensors
        dq, dk, dv, dc = _pka._bwd(q, k, v, o, den, do, ctx.num_groups, ctx.scale, ctx.score, c=c, cu=cu)
        return dq, dk, dv, dc, None, None, None, None


def _packed_ok(q, k, v, num_groups, score, c, nseq) -> bool:
    """True when the tensor-core kernels take the packed documents as they lie."""
    if _pka.ALGO in ("simt", "tc_gram") or q.dtype not in (torch.bfloat16, torch.float16):
        return False
    if k.dtype != q.dtype or v.dtype != q.dtype or not q.is_cuda or nseq < 1:
        return False
    a = _lib.AttnFwdArgs(dtype=_lib.DTYPE[q.dtype], B=1, T=max(q.shape[1], 1), H=k.shape[2], HQ=q.shape[2],
                         D=q.shape[-1], Dv=v.shape[-1], M=num_groups, score=_lib.SCORE[score],
                         algo=_lib.ALGO["tc"], scale=1.0, c=None if c is None else 16, cu_seqlens=1, num_seqs=nseq)
    return _lib.lib().kata_attn_algo(a) == _lib.ALGO["tc"]


def parallel_kata_attn_varlen(q, k, v, cu_seqlens, num_groups=4, scale=None, score="concat", c=None,
                              max_seqlen=None):
    """Causal KATA-SPD attention over packed documents.

    q (1, T_total, HQ, D), k (1, T_total, H, D), v (1, T_total, H, Dv); ``cu_seqlens`` (N+1) int;
    ``score`` "concat" or "sum"; ``c`` (1, T_total, HQ) fp32 cumulative log-decay (concat score,
    per document: the decay factor only ever compares tokens of one document).  ``max_seqlen``
    (the longest document) avoids a device-to-host read of ``cu_seqlens``; with a device-resident
    ``cu_seqlens`` and ``max_seqlen`` given, the caller guarantees that cu_seqlens starts at 0, is
    non-decreasing, ends at T_total and has no document longer than max_seqlen (a CPU cu_seqlens
    is always checked).  Returns o
    (1, T_total, HQ, Dv) in v's dtype; autograd gives dq, dk, dv (and dc).
    """
    if q.dim() != 4 or q.shape[0] != 1:
        raise ValueError(f"packed inputs are (1, T_total, H, D); got q {tuple(q.shape)}")
    if score not in ("concat", "sum"):
        raise ValueError(f"score must be 'concat' or 'sum', got {score!r}")
    if c is not None and score != "concat":
        raise ValueError("decay pairs with the concat score only")
    if max_seqlen is None or cu_seqlens.device.type == "cpu":
        # validate cu_seqlens on the host whenever that costs no device-to-host read: start at 0,
        # non-decreasing, total == q.shape[1], and no document longer than max_seqlen (a shorter
        # max_seqlen would make documents collide in the padded batch)
        cpu = cu_seqlens.cpu().to(torch.int64)
        if cpu.dim() != 1 or cpu.numel() < 2:
            raise ValueError("cu_seqlens must be 1-D with at least two entries")
        lens = cpu[1:] - cpu[:-1]
        if int(cpu[0]) != 0 or bool((lens < 0).any()):
            raise ValueError("cu_seqlens must start at 0 and be non-decreasing")
        if int(cpu[-1]) != q.shape[1]:
            raise ValueError(f"cu_seqlens covers {int(cpu[-1])} tokens, q has {q.shape[1]}")
        if max_seqlen is not None and int(lens.max()) > int(max_seqlen):
            raise ValueError(f"max_seqlen {max_seqlen} is below the longest document ({int(lens.max())})")
    nseq = cu_seqlens.numel() - 1
    if q.shape[1] > 0 and _packed_ok(q, k, v, num_groups, score, c, nseq):
        cu = cu_seqlens.to(device=q.device, dtype=torch.int32).contiguous()
        return _PackedKataFunction.apply(q, k, v, c, cu, num_groups, scale, score)
    dst, N, T_max = varlen_index(cu_seqlens.to(q.device), max_seqlen, total=q.shape[1])
    qp, kp, vp = (pack_rows(x, dst, N, T_max) for x in (q, k, v))
    if c is not None:
        o = parallel_kata_attn_decay(qp, kp, vp, pack_rows(c, dst, N, T_max), num_groups=num_groups, scale=scale)
    elif score == "sum":
        o = parallel_kata_attn_sum(qp, kp, vp, num_groups=num_groups, scale=scale)
    else:
        o = parallel_kata_attn(qp, kp, vp, num_groups=num_groups, scale=scale)
    return unpack_rows(o, dst)
