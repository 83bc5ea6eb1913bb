"""CPU oracle for the KATA-SPD attention hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import this module, and only as the checker or the timed CPU baseline; the product path
(``linatt_b200``) never calls it.

Everything is a float64 NumPy restatement of the reference's algorithm, one (batch, head) slice
at a time so memory stays O(T^2 * parts).  Parity is pinned: ``tests/golden/make_golden.py``
runs the reference's own PyTorch functions (and its Triton forward kernels under the Triton CPU
interpreter) on seeded inputs and stores their outputs; ``tests/test_oracle.py`` checks this
module against every one of those fixtures.

Reference map (paths relative to the ayghri/linatt checkout):
  attn_fwd      -- kata/kernels/parallel_kata.py:10-197 (K1, concat) and :202-345 (K2, sum);
                   den <= 0 -> divide by 1 (:193-196); decay factor exp(min(c_t-c_s,0)) (:128-134)
  attn_bwd      -- kata/parallel_kata_attn.py:49-146 (concat), :579-653 (sum); decay gradients
                   including dc follow autograd through _kata_decay_ref (:291-310, :329-347)
  augment_offset-- kata/layer.py:268-282
"""

from __future__ import annotations

import numpy as np


def _parts(M: int, score: str):
    if score == "concat":
        return [(g, g) for g in range(M)]
    if score == "sum":
        return [(a, b) for a in range(M) for b in range(M)]
    raise ValueError(score)


def _head_scores(qh, kh, M, scale, score):
    """qh (T,D), kh (T,D) float64 -> list of qk_p (T,T) with qk_p = scale * <q_a, k_b>."""
    T, D = qh.shape
    E = D // M
    out = []
    for a, b in _parts(M, score):
        out.append(scale * (qh[:, a * E:(a + 1) * E] @ kh[:, b * E:(b + 1) * E].T))
    return out


def _decay(ch):
    """ch (T,) -> (dec (T,T), active (T,T)) with dec = exp(min(c_t - c_s, 0))."""
    x = ch[:, None] - ch[None, :]
    return np.exp(np.minimum(x, 0.0)), (x <= 0.0)


def attn_fwd(q, k, v, M, scale=None, score="concat", c=None):
    """Causal normalised KATA-SPD attention forward.

    q (B,T,HQ,D), k (B,T,H,D), v (B,T,H,Dv), optional c (B,T,HQ) -> o (B,T,HQ,Dv), den (B,T,HQ).
    """
    q, k, v = (np.asarray(x, dtype=np.float64) for x in (q, k, v))
    B, T, HQ, D = q.shape
    H = k.shape[2]
    G = HQ // H
    Dv = v.shape[-1]
    if scale is None:
        scale = 1.0 / np.sqrt(D // M)
    tri = np.tril(np.ones((T, T)))
    o = np.zeros((B, T, HQ, Dv))
    den = np.zeros((B, T, HQ))
    for b in range(B):
        for hq in range(HQ):
            h = hq // G
            parts = _head_scores(q[b, :, hq], k[b, :, h], M, scale, score)
            A = sum(p * p for p in parts) * tri
            if c is not None:
                A = A * _decay(np.asarray(c, dtype=np.float64)[b, :, hq])[0]
            dn = A.sum(1)
            o[b, :, hq] = (A @ v[b, :, h]) / np.where(dn > 0, dn, 1.0)[:, None]
            den[b, :, hq] = dn
    return o, den


def attn_bwd(q, k, v, do, M, scale=None, score="concat", c=None):
    """Gradients of sum(o * do) w.r.t. q, k, v (and c) for ``attn_fwd``.

    Closed form of kata/parallel_kata_attn.py:49-146 (dA = (dO.v - delta)/den; d(qk_p) = 2 qk_p dA;
    dv = P^T dO), :579-653 for the sum score, and the c-gradient that autograd produces through
    _kata_decay_ref: dc_t = sum_s G[t,s] - sum_t' G[t',t], G = dA * A on pairs with c_t-c_s <= 0.
    Returns (dq, dk, dv, dc) with dc None when c is None.
    """
    q, k, v, do = (np.asarray(x, dtype=np.float64) for x in (q, k, v, do))
    B, T, HQ, D = q.shape
    H = k.shape[2]
    G = HQ // H
    Dv = v.shape[-1]
    E = D // M
    if scale is None:
        scale = 1.0 / np.sqrt(E)
    tri = np.tril(np.ones((T, T)))
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    dc = np.zeros((B, T, HQ)) if c is not None else None
    pl = _parts(M, score)
    for b in range(B):
        for hq in range(HQ):
            h = hq // G
            qh, kh, vh, doh = q[b, :, hq], k[b, :, h], v[b, :, h], do[b, :, hq]
            parts = _head_scores(qh, kh, M, scale, score)
            A0 = sum(p * p for p in parts) * tri
            dec = np.ones((T, T))
            act = np.ones((T, T), dtype=bool)
            if c is not None:
                dec, act = _decay(np.asarray(c, dtype=np.float64)[b, :, hq])
            A = A0 * dec
            dn = A.sum(1)
            rden = 1.0 / np.where(dn > 0, dn, 1.0)
            P = A * rden[:, None]
            o = P @ vh
            delta = (o * doh).sum(1)
            dA = (doh @ vh.T - delta[:, None]) * rden[:, None] * tri
            dv[b, :, h] += P.T @ doh
            for (a, bb), qk in zip(pl, parts):
                W = 2.0 * scale * qk * dec * dA
                dq[b, :, hq, a * E:(a + 1) * E] += W @ kh[:, bb * E:(bb + 1) * E]
                dk[b, :, h, bb * E:(bb + 1) * E] += W.T @ qh[:, a * E:(a + 1) * E]
            if c is not None:
                Gm = dA * A * act * tri
                dc[b, :, hq] = Gm.sum(1) - Gm.sum(0)
    return dq, dk, dv, dc


def attn_tail_window(qh, kh, vh, doh, M, w, scale=None, chunk=8192):
    """Exact concat-score forward and backward restricted to the last ``w`` tokens of one long head.

    qh, kh, vh, doh (T, D/Dv) for one (batch, head).  Row t of o, den, delta and dq depends on row t
    against every key s <= t, and the key rows s >= T - w of dk and dv depend only on queries t >= s,
    all inside the window; so this is exact for the window at any T while memory stays
    O(w * chunk).  Same formulas as ``attn_fwd`` / ``attn_bwd`` (kata/parallel_kata_attn.py:49-146).
    Returns dict o, den, dq (rows T-w..T-1) and dk, dv (key rows T-w..T-1), float64.
    """
    qh, kh, vh, doh = (np.asarray(x, dtype=np.float64) for x in (qh, kh, vh, doh))
    T, D = qh.shape
    E = D // M
    if scale is None:
        scale = 1.0 / np.sqrt(E)
    t0 = T - w
    qr, dor = qh[t0:], doh[t0:]
    rows = np.arange(t0, T)[:, None]

    def blocks():
        for s0 in range(0, T, chunk):
            s1 = min(T, s0 + chunk)
            qk = [scale * (qr[:, g * E:(g + 1) * E] @ kh[s0:s1, g * E:(g + 1) * E].T) for g in range(M)]
            mask = (np.arange(s0, s1)[None, :] <= rows)
            yield s0, s1, qk, sum(p * p for p in qk) * mask, mask

    den = np.zeros(w)
    num = np.zeros((w, vh.shape[1]))
    for s0, s1, _, A, _ in blocks():
        den += A.sum(1)
        num += A @ vh[s0:s1]
    rden = 1.0 / np.where(den > 0, den, 1.0)
    o = num * rden[:, None]
    delta = (o * dor).sum(1)
    dq = np.zeros((w, D))
    dk = np.zeros((w, D))
    dv = np.zeros((w, vh.shape[1]))
    for s0, s1, qk, A, mask in blocks():
        dA = (dor @ vh[s0:s1].T - delta[:, None]) * rden[:, None] * mask
        for g in range(M):
            W = 2.0 * scale * qk[g] * dA
            dq[:, g * E:(g + 1) * E] += W @ kh[s0:s1, g * E:(g + 1) * E]
            if s1 > t0:  # key rows inside the window
                a = max(s0, t0)
                dk[a - t0:s1 - t0, g * E:(g + 1) * E] += W[:, a - s0:].T @ qr[:, g * E:(g + 1) * E]
        if s1 > t0:
            a = max(s0, t0)
            dv[a - t0:s1 - t0] += (A[:, a - s0:] * rden[:, None]).T @ dor
    return {"o": o, "den": den, "dq": dq, "dk": dk, "dv": dv}


def augment_offset(q, k, off, M):
    """Offset gate packing (kata/layer.py:268-282): append off_t to each q group and 1 to each k
    group, zero-pad every group to Ep = max(16, 2**bit_length(E)); returns (q_in, k_in)."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    off = np.asarray(off, dtype=np.float64)
    B, T, H, D = q.shape
    E = D // M
    Ep = max(16, 1 << int(E).bit_length())

    def pack(x, col):
        xg = x.reshape(B, T, H, M, E)
        cc = np.broadcast_to(col[..., None, None], (B, T, H, M, 1))
        z = np.zeros((B, T, H, M, Ep - E - 1))
        return np.concatenate([xg, cc, z], axis=-1).reshape(B, T, H, M * Ep)

    return pack(q, off), pack(k, np.ones_like(off))


def rel_l2(x, ref) -> float:
    """||x - ref||_2 / ||ref||_2 in float64 (0 when both vanish)."""
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    n = np.linalg.norm(ref)
    d = np.linalg.norm(x - ref)
    return float(d / n) if n > 0 else float(d)
