"""Golden fixtures for the gated delta rule (third-party arithmetic: flash-linear-attention,
``fla``; the reference pins 0.5.0, 0.5.1 is what this was generated with), from fla's own PyTorch
references, in a container where ``fla`` is importable:

    python tests/golden/make_golden_gdn.py

``fla.ops.gated_delta_rule.naive.naive_recurrent_gated_delta_rule`` (naive.py:13-60) gives o, the
final state and, through torch autograd, the gradients of sum(o * dO) + sum(ht * dht) with respect
to q, k, v, g, beta and the initial state; ``naive_chunk_gated_delta_rule`` (naive.py:67-160)
gives a second forward witness of the chunked form.  Variable-length fixtures concatenate
per-sequence runs (what ``cu_seqlens`` means).  All computed in float32 on CPU, stored as float32
in ``tests/golden/gdn_golden.npz``.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F
from fla.ops.gated_delta_rule.naive import naive_chunk_gated_delta_rule, naive_recurrent_gated_delta_rule

OUT = Path(__file__).resolve().parent / "gdn_golden.npz"


def draw(seed, B, T, H, K, V, h0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, K, generator=g)
    k = F.normalize(torch.randn(B, T, H, K, generator=g), dim=-1)
    v = torch.randn(B, T, H, V, generator=g)
    beta = torch.sigmoid(torch.randn(B, T, H, generator=g))
    gate = -F.softplus(torch.randn(B, T, H, generator=g))
    do = torch.randn(B, T, H, V, generator=g)
    N = B
    s0 = torch.randn(N, H, K, V, generator=g) * 0.1 if h0 else None
    dht = torch.randn(N, H, K, V, generator=g) * 0.1
    return q, k, v, beta, gate, do, s0, dht


def run_case(out, name, seed, B, T, H, K, V, h0, cu=None):
    q, k, v, beta, gate, do, s0, dht = draw(seed, B, T, H, K, V, h0)
    if cu is not None:
        s0 = torch.randn(len(cu) - 1, H, K, V, generator=torch.Generator().manual_seed(seed + 1)) * 0.1 if h0 else None
        dht = torch.randn(len(cu) - 1, H, K, V, generator=torch.Generator().manual_seed(seed + 2)) * 0.1
    leaves = [x.clone().requires_grad_(True) for x in (q, k, v, gate, beta)]
    h0l = s0.clone().requires_grad_(True) if s0 is not None else None
    ql, kl, vl, gl, bl = leaves
    if cu is None:
        o, ht = naive_recurrent_gated_delta_rule(ql, kl, vl, bl, gl, initial_state=h0l, output_final_state=True)
    else:
        os_, hs = [], []
        for i in range(len(cu) - 1):
            a, b = cu[i], cu[i + 1]
            oi, hi = naive_recurrent_gated_delta_rule(ql[:, a:b], kl[:, a:b], vl[:, a:b], bl[:, a:b], gl[:, a:b],
                                                      initial_state=None if h0l is None else h0l[i:i + 1],
                                                      output_final_state=True)
            os_.append(oi)
            hs.append(hi)
        o, ht = torch.cat(os_, 1), torch.cat(hs, 0)
    loss = (o * do).sum() + (ht * dht).sum()
    grads = torch.autograd.grad(loss, leaves + ([h0l] if h0l is not None else []))
    rec = dict(q=q, k=k, v=v, beta=beta, g=gate, do=do, dht=dht, o=o.detach(), ht=ht.detach(),
               dq=grads[0], dk=grads[1], dv=grads[2], dg=grads[3], dbeta=grads[4])
    if s0 is not None:
        rec.update(h0=s0, dh0=grads[5])
    if cu is None:
        oc, hc = naive_chunk_gated_delta_rule(q, k, v, gate, beta, chunk_size=64, initial_state=s0,
                                              output_final_state=True)
        rec.update(o_chunk=oc, ht_chunk=hc)
    else:
        rec["cu_seqlens"] = torch.tensor(cu, dtype=torch.int64)
    for key, val in rec.items():
        out[f"{name}/{key}"] = val.numpy().astype(np.int64 if key == "cu_seqlens" else np.float32)
    out[f"{name}/meta"] = np.array([B, T, H, K, V, int(h0)], dtype=np.int64)


def main():
    torch.set_num_threads(8)
    out = {}
    run_case(out, "basic", 1, 2, 100, 2, 32, 16, True)
    run_case(out, "chunk_t128", 2, 1, 128, 2, 64, 64, False)
    run_case(out, "varlen", 3, 1, 160, 2, 32, 32, True, cu=[0, 37, 100, 160])
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1e6:.2f} MB)")


if __name__ == "__main__":
    main()
