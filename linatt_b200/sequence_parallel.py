"""Sequence-parallel causal KATA-SPD attention (concat score) over a contiguous split of T.

No counterpart exists in the reference: ``kata/parallel_kata_attn.py`` is "parallel" over T within
one GPU (its docstring, :1-22).  This module is the long-context multi-GPU path: rank r of a
process group holds tokens [r*T/R, (r+1)*T/R) of every head and computes

    o_t = (n_t + psi(q_t)^T P) / D_t',   D_t = d_t + psi(q_t)^T z,   x' = x if x > 0 else 1

where n_t / d_t are the shard-local causal numerator / denominator (the flash kernels of
``linatt_b200.parallel_kata_attn``), psi(x)[g,a,b] = scale * x_{g,a} x_{g,b} is the quadratic feature
map with A[t,s] = psi(q_t).psi(k_s), and [P | z] = sum over earlier shards of psi(k_s) [v_s | 1]
(an F x (Dv+1) state per head, F = M E^2).  The only exchange is that state: an exclusive prefix
over ranks in the forward and an exclusive suffix of its gradient in the backward, each an NCCL
all-gather issued before the shard-local attention kernel so that it overlaps it.

The shard-local backward is the single-GPU kernel run with the final o and D: its
dA = (dO.v - <dO,o>) / D is then exactly the local block of the full gradient.  The F-wide
contractions (the state psi(K)^T [V|1], the prefix term psi(Q) P, their gradients psi(Q)^T W1,
psi(K) dS and the contractions of W1 P^T, [V|1] dS^T back to dq, dk) are tcgen05 kernels of
``libkata_b200.so`` that form psi tiles in shared memory (``kata_sp_state`` / ``_apply`` /
``_grad``); psi is never written to global memory.  States are kept transposed, (B*H, ldw, F).
Head widths outside those kernels' envelope (E = D/M not in {16, 32}) take the earlier route:
materialised psi (``kata_sp_features``) and bf16 GEMMs with fp32 output (torch.bmm).
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from . import _lib
from . import parallel_kata_attn as pka

__all__ = ["sp_kata_attn", "SPKataAttnFunction", "exclusive_prefix_sum", "exclusive_suffix_sum",
           "gather_states", "sp_forward_local", "sp_forward_combine", "sp_backward_prep", "sp_backward",
           "sp_backward_local", "sp_backward_cross", "sp_emulate"]


# ------------------------------------------------------------------------------------------------
# exchange (host logic; any backend)
# ------------------------------------------------------------------------------------------------
class _Gathered:
    def __init__(self, bufs, work, world):
        self.bufs, self.work, self.world = bufs, work, world

    def wait(self) -> torch.Tensor:
        if self.work is not None:
            self.work.wait()
        return self.bufs if isinstance(self.bufs, torch.Tensor) else torch.stack(self.bufs)


def gather_states(x: torch.Tensor, group=None, async_op: bool = False) -> _Gathered:
    """All ranks' ``x`` stacked along a new leading dim (rank order); ``.wait()`` returns it."""
    world = dist.get_world_size(group)
    x = x.contiguous()
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world,) + tuple(x.shape), dtype=x.dtype, device=x.device)
        work = dist.all_gather_into_tensor(out, x, group=group, async_op=async_op)
        return _Gathered(out, work, world)
    outs = [torch.empty_like(x) for _ in range(world)]
    work = dist.all_gather(outs, x, group=group, async_op=async_op)
    return _Gathered(outs, work, world)


def exclusive_prefix_sum(stacked: torch.Tensor, rank: int) -> torch.Tensor | None:
    """sum_{r < rank} stacked[r]  (None for rank 0)."""
    return stacked[:rank].sum(0) if rank > 0 else None


def exclusive_suffix_sum(stacked: torch.Tensor, rank: int) -> torch.Tensor | None:
    """sum_{r > rank} stacked[r]  (None for the last rank)."""
    return stacked[rank + 1:].sum(0) if rank + 1 < stacked.shape[0] else None


# ------------------------------------------------------------------------------------------------
# shard-local pieces (GPU)
# ------------------------------------------------------------------------------------------------
def _ldw(Dv: int) -> int:
    return (Dv + 1 + 7) // 8 * 8  # [v | 1 | zero pad] width, a multiple of 8 for the GEMMs


def _features(x, M, scale):
    x = x.contiguous()  # the kernel reads dense (B, T, H, D) rows
    B, T, H, D = x.shape
    E = D // M
    R = torch.empty(B * H, T, M * E * E, device=x.device, dtype=torch.bfloat16)
    _lib.check(_lib.lib().kata_sp_features(x.data_ptr(), R.data_ptr(), _lib.DTYPE[x.dtype], B, T, H, D, M,
                                           float(scale), _lib.stream_handle(x.device)), "kata_sp_features")
    return R


def _contract(G, x, dx, M, scale):
    x = x.contiguous()  # dx is a dense fp32 (B, T, H, D) buffer made by the caller
    B, T, H, D = x.shape
    _lib.check(_lib.lib().kata_sp_contract(G.data_ptr(), x.data_ptr(), dx.data_ptr(), _lib.DTYPE[x.dtype], B, T, H,
                                           D, M, 2.0 * float(scale), 1, _lib.stream_handle(x.device)),
               "kata_sp_contract")


def _v1(v, ldw):
    B, T, H, Dv = v.shape
    out = torch.zeros(B, H, T, ldw, device=v.device, dtype=torch.bfloat16)
    out[..., :Dv] = v.permute(0, 2, 1, 3)
    out[..., Dv] = 1.0
    return out.view(B * H, T, ldw)


def _scale(D, M, scale):
    return 1.0 / math.sqrt(D // M) if scale is None else float(scale)


def _tc_ok(x, num_groups, ldw):
    """The feature-contraction kernels cover 16-bit inputs with E = D/M in {16, 32}, D in {64, 128}."""
    D = x.shape[-1]
    return (x.dtype in (torch.bfloat16, torch.float16) and D in (64, 128) and D % num_groups == 0
            and D // num_groups in (16, 32) and ldw <= 144)


def _state(x, W, num_groups, scale):
    """S^T (B*H, ldw, F) fp32 = (psi(x)^T W)^T for x (B,T,H,D) and W (B*H, T, ldw) bf16."""
    x = x.contiguous()
    B, T, H, D = x.shape
    ldw = W.shape[-1]
    F = num_groups * (D // num_groups) ** 2
    if not _tc_ok(x, num_groups, ldw):
        R = _features(x, num_groups, scale)
        return torch.bmm(W.transpose(1, 2), R, out_dtype=torch.float32)
    S = torch.empty(B * H, ldw, F, device=x.device, dtype=torch.float32)
    _lib.check(_lib.lib().kata_sp_state(x.data_ptr(), W.data_ptr(), S.data_ptr(), _lib.DTYPE[x.dtype], B, T, H, 1, D,
                                        num_groups, _lib.SCORE["concat"], ldw, float(scale), 1, ldw,
                                        _lib.status_word(x.device).data_ptr(), _lib.stream_handle(x.device)),
               "kata_sp_state")
    return S


def _apply(x, Pt, num_groups, scale, dv=None):
    """Y (B*H, T, ldw) fp32 = psi(x) P for P^T = Pt (B*H, ldw, F) bf16; with ``dv`` (B,T,H,Dv) fp32,
    adds Y[..., :Dv] into it instead (returns None)."""
    x = x.contiguous()
    B, T, H, D = x.shape
    ldw = Pt.shape[1]
    if not _tc_ok(x, num_groups, ldw):
        Y = torch.bmm(_features(x, num_groups, scale), Pt.transpose(1, 2), out_dtype=torch.float32)
        if dv is None:
            return Y
        Dv = dv.shape[-1]
        dv += Y[..., :Dv].reshape(B, H, T, Dv).permute(0, 2, 1, 3)
        return None
    Y = dv if dv is not None else torch.empty(B * H, T, ldw, device=x.device, dtype=torch.float32)
    _lib.check(_lib.lib().kata_sp_apply(x.data_ptr(), Pt.data_ptr(), Y.data_ptr(), _lib.DTYPE[x.dtype], B, T, H, 1, D,
                                        num_groups, ldw, float(scale), int(dv is not None),
                                        dv.shape[-1] if dv is not None else 0, _lib.status_word(x.device).data_ptr(),
                                        _lib.stream_handle(x.device)), "kata_sp_apply")
    return None if dv is not None else Y


def _grad(W, Pt, x, dx, num_groups, scale):
    """dx (B,T,H,D) fp32 += the gradient through psi(x) of <W P^T, psi(x)> (factor 2 scale)."""
    x = x.contiguous()
    B, T, H, D = x.shape
    ldw = W.shape[-1]
    if not _tc_ok(x, num_groups, ldw):
        G = torch.bmm(W, Pt)  # (B*H, T, F) bf16
        _contract(G, x, dx, num_groups, scale)
        return
    _lib.check(_lib.lib().kata_sp_grad(W.data_ptr(), Pt.data_ptr(), x.data_ptr(), dx.data_ptr(), _lib.DTYPE[x.dtype],
                                       B, T, H, D, num_groups, ldw, 2.0 * float(scale),
                                       _lib.status_word(x.device).data_ptr(), _lib.stream_handle(x.device)),
               "kata_sp_grad")


def sp_forward_local(q, k, v, num_groups, scale, want_state=True):
    """Shard-local causal attention and this shard's state contribution.
    Returns (o_local, den_local, S) with S^T = (psi(K)^T [V | 1])^T (B*H, ldw, F) fp32 (None if not wanted)."""
    scale = _scale(q.shape[-1], num_groups, scale)
    S = _state(k, _v1(v, _ldw(v.shape[-1])), num_groups, scale) if want_state else None
    o_loc, den = pka._fwd(q, k, v, num_groups, scale, "concat")
    return o_loc, den, S


def sp_forward_combine(q, o_loc, den_loc, P, num_groups, scale):
    """Final (o, D) of a shard from its local result and the prefix state P^T (None: first shard)."""
    if P is None:
        return o_loc, den_loc
    scale = _scale(q.shape[-1], num_groups, scale)
    B, T, H, Dv = o_loc.shape
    XY = _apply(q, P.to(torch.bfloat16), num_groups, scale)
    o = torch.empty_like(o_loc)
    D = torch.empty_like(den_loc)
    _lib.check(_lib.lib().kata_sp_combine(o_loc.data_ptr(), den_loc.data_ptr(), XY.data_ptr(), o.data_ptr(),
                                          D.data_ptr(), _lib.DTYPE[o_loc.dtype], B, T, H, Dv, XY.shape[-1],
                                          _lib.stream_handle(q.device)), "kata_sp_combine")
    return o, D


def sp_backward_prep(q, o, D, do, num_groups, scale, want_dP=True):
    """W1 = [dO/D' | -<dO,o>/D' | 0] and this shard's gradient of its prefix state, dP^T with
    dP = psi(Q)^T W1."""
    B, T, H, Dv = o.shape
    ldw = _ldw(Dv)
    W1 = torch.empty(B * H, T, ldw, device=o.device, dtype=torch.bfloat16)
    _lib.check(_lib.lib().kata_sp_bwd_prep(o.data_ptr(), do.data_ptr(), D.data_ptr(), W1.data_ptr(),
                                           _lib.DTYPE[o.dtype], B, T, H, Dv, ldw, _lib.stream_handle(o.device)),
               "kata_sp_bwd_prep")
    dP = None
    if want_dP:
        dP = _state(q, W1, num_groups, _scale(q.shape[-1], num_groups, scale))
    return W1, dP


def sp_backward_cross(q, k, v, W1, P, dS, dq, dk, dv, num_groups, scale):
    """Adds to the fp32 dq, dk, dv of a shard the prefix term (through P^T, the bf16 prefix state)
    and the state term (through dS^T = the sum of later shards' dP^T)."""
    scale = _scale(q.shape[-1], num_groups, scale)
    if P is not None:
        _grad(W1, P.to(torch.bfloat16), q, dq, num_groups, scale)
    if dS is not None:
        dSb = dS.to(torch.bfloat16)
        _apply(k, dSb, num_groups, scale, dv=dv)
        _grad(_v1(v, W1.shape[-1]), dSb, k, dk, num_groups, scale)


def sp_backward_local(q, k, v, o, D, do, num_groups, scale):
    """The shard-local block of the gradient: the flash backward run with the final o and D."""
    dq, dk, dv, _ = pka._bwd(q, k, v, o, D, do, num_groups, _scale(q.shape[-1], num_groups, scale), "concat")
    return dq.float(), dk.float(), dv.float()


def sp_backward(q, k, v, o, D, do, W1, P, dS, num_groups, scale):
    """dq, dk, dv (fp32) of a shard: local block + prefix term + state term."""
    dq, dk, dv = sp_backward_local(q, k, v, o, D, do, num_groups, scale)
    sp_backward_cross(q, k, v, W1, P, dS, dq, dk, dv, num_groups, scale)
    return dq, dk, dv


def sp_emulate(q, k, v, do, R, num_groups, scale=None):
    """Forward + backward of the sequence-parallel algorithm over R shards of the sequence, run one
    after another on the current device, with the exchange (exclusive prefix of the states, exclusive
    suffix of their gradients) formed locally.  Same kernels and arithmetic as R ranks over NCCL;
    for checking the algorithm and profiling its kernels on one GPU.  Returns (o, D, dq, dk, dv)."""
    qs, ks, vs, dos = (x.chunk(R, dim=1) for x in (q, k, v, do))
    loc = [sp_forward_local(qs[r], ks[r], vs[r], num_groups, scale, want_state=r < R - 1) for r in range(R)]
    states = [S for _, _, S in loc[:-1]]
    outs, dens, prefixes = [], [], []
    for r in range(R):
        P = sum(states[:r]) if r > 0 else None
        o, D = sp_forward_combine(qs[r], loc[r][0], loc[r][1], P, num_groups, scale)
        outs.append(o)
        dens.append(D)
        prefixes.append(P.to(torch.bfloat16) if P is not None else None)
    preps = [sp_backward_prep(qs[r], outs[r], dens[r], dos[r].contiguous(), num_groups, scale, want_dP=r > 0)
             for r in range(R)]
    grads = []
    for r in range(R):
        later = [preps[j][1] for j in range(r + 1, R)]
        dS = sum(later) if later else None
        grads.append(sp_backward(qs[r], ks[r], vs[r], outs[r], dens[r], dos[r].contiguous(), preps[r][0],
                                 prefixes[r], dS, num_groups, scale))
    cat = lambda xs: torch.cat(xs, dim=1)  # noqa: E731
    return (cat(outs), cat(dens), cat([g[0] for g in grads]), cat([g[1] for g in grads]),
            cat([g[2] for g in grads]))


# ------------------------------------------------------------------------------------------------
# autograd op
# ------------------------------------------------------------------------------------------------
class SPKataAttnFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, num_groups, scale, group):
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        q, k, v = (x.contiguous() for x in (q, k, v))
        scale = _scale(q.shape[-1], num_groups, scale)
        B, T, H, Dv = v.shape
        F = num_groups * (q.shape[-1] // num_groups) ** 2
        last = rank == world - 1
        # state first, so that its all-gather overlaps the shard-local attention kernel
        if not last:
            S = _state(k, _v1(v, _ldw(Dv)), num_groups, scale)
        else:  # the last shard's state feeds nobody
            S = torch.zeros(B * H, _ldw(Dv), F, device=q.device, dtype=torch.float32)
        pending = gather_states(S, group, async_op=True)
        o_loc, den_loc = pka._fwd(q, k, v, num_groups, scale, "concat")
        P = exclusive_prefix_sum(pending.wait(), rank)
        o, D = sp_forward_combine(q, o_loc, den_loc, P, num_groups, scale)
        Pb = P.to(torch.bfloat16) if P is not None else None
        ctx.save_for_backward(q, k, v, o, D, Pb)
        ctx.num_groups, ctx.scale, ctx.group, ctx.rank, ctx.world = num_groups, scale, group, rank, world
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, D, Pb = ctx.saved_tensors
        do = do.to(o.dtype).contiguous()
        W1, dP = sp_backward_prep(q, o, D, do, ctx.num_groups, ctx.scale, want_dP=ctx.rank > 0)
        if dP is None:  # the first shard's prefix gradient feeds nobody
            F = ctx.num_groups * (q.shape[-1] // ctx.num_groups) ** 2
            dP = torch.zeros(W1.shape[0], W1.shape[-1], F, device=q.device, dtype=torch.float32)
        pending = gather_states(dP, ctx.group, async_op=True)
        dq, dk, dv = sp_backward_local(q, k, v, o, D, do, ctx.num_groups, ctx.scale)
        dS = exclusive_suffix_sum(pending.wait(), ctx.rank)
        sp_backward_cross(q, k, v, W1, Pb, dS, dq, dk, dv, ctx.num_groups, ctx.scale)
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), None, None, None


def sp_kata_attn(q, k, v, num_groups=4, scale=None, group=None):
    """Causal concat-score KATA-SPD attention of a sequence split contiguously over the ranks of
    ``group`` (rank order = sequence order).  q, k, v: this rank's (B, T/R, H, D) shard, time-major;
    returns this rank's shard of o.  With one rank it is ``parallel_kata_attn``."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return pka.parallel_kata_attn(q, k, v, num_groups=num_groups, scale=scale)
    if q.shape[2] != k.shape[2]:
        raise NotImplementedError("sequence-parallel path: q and k must have the same number of heads")
    return SPKataAttnFunction.apply(q, k, v, num_groups, scale, group)
