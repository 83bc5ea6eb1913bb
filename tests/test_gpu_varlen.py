"""GPU parity of the packed-sequence API: outputs and gradients of parallel_kata_attn_varlen over
packed documents equal one flash call per document (bf16 / fp16: rel-L2 <= 1e-2, fp32: <= 1e-5), for
the concat and sum scores, the decayed form and GQA, with ragged, empty and length-1 documents.
16-bit inputs take the tensor-core kernels' packed-document form (no padding), with or without
decay; fp32 takes the padded batch.  The two forms are also compared with each other."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle.kata_oracle import rel_l2

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return rel_l2(a.detach().float().cpu().numpy(), b.detach().float().cpu().numpy())


@pytest.mark.parametrize("lens,HQ,H,D,M,score,dtype,decay", [
    ([100, 1, 256, 63], 2, 2, 128, 4, "concat", torch.bfloat16, False),
    ([70, 0, 129], 4, 2, 128, 2, "concat", torch.bfloat16, False),
    ([40, 97, 1], 2, 2, 64, 2, "concat", torch.float32, False),
    ([65, 130, 7], 2, 2, 64, 4, "sum", torch.bfloat16, False),
    ([90, 33, 200], 2, 2, 128, 2, "concat", torch.bfloat16, True),
    ([128, 129, 127, 1, 256], 2, 2, 64, 4, "concat", torch.bfloat16, False),
    ([5 + 11 * i for i in range(40)], 2, 1, 64, 4, "concat", torch.bfloat16, False),
    ([300, 77], 2, 2, 128, 4, "concat", torch.float16, False),
    ([1000], 2, 2, 128, 1, "concat", torch.bfloat16, False),
])
def test_varlen_matches_per_document_calls(lens, HQ, H, D, M, score, dtype, decay):
    from linatt_b200.parallel_kata_attn import parallel_kata_attn, parallel_kata_attn_decay, parallel_kata_attn_sum
    from linatt_b200.varlen import parallel_kata_attn_varlen

    T = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    g = torch.Generator().manual_seed(T + D + M)
    q = (torch.randn(1, T, HQ, D, generator=g) / D ** 0.5).to(dtype).cuda()
    k = F.normalize(torch.randn(1, T, H, D, generator=g), dim=-1).to(dtype).cuda()
    v = torch.randn(1, T, H, D, generator=g).to(dtype).cuda()
    do = torch.randn(1, T, HQ, D, generator=g).to(dtype).cuda()
    c = -F.softplus(torch.randn(1, T, HQ, generator=g)).cumsum(1).cuda() if decay else None

    leaves = [x.clone().requires_grad_(True) for x in (q, k, v)] + ([c.clone().requires_grad_(True)] if decay else [])
    o = parallel_kata_attn_varlen(*leaves[:3], cu.cuda(), num_groups=M, score=score, c=leaves[3] if decay else None)
    o.backward(do)

    tol = 1e-5 if dtype == torch.float32 else 1e-2
    starts = cu.tolist()
    for n in range(len(lens)):
        s, e = starts[n], starts[n + 1]
        if s == e:
            continue
        part = [x[:, s:e].detach().clone().requires_grad_(True) for x in (q, k, v)]
        if decay:
            part.append(c[:, s:e].detach().clone().requires_grad_(True))
            ref = parallel_kata_attn_decay(*part, num_groups=M)
        elif score == "sum":
            ref = parallel_kata_attn_sum(*part, num_groups=M)
        else:
            ref = parallel_kata_attn(*part, num_groups=M)
        ref.backward(do[:, s:e])
        assert _rel(o[:, s:e], ref) < tol, f"doc {n} o"
        for i, name in enumerate(["dq", "dk", "dv", "dc"][:len(part)]):
            assert _rel(leaves[i].grad[:, s:e], part[i].grad) < tol, f"doc {n} {name}"


@pytest.mark.parametrize("lens,HQ,H,D,M,score,decay", [
    ([100, 1, 256, 63, 0, 130], 4, 2, 128, 4, "concat", False),
    ([65, 130, 7, 300], 2, 2, 64, 4, "sum", False),
    ([3 + 7 * i for i in range(70)], 2, 2, 64, 2, "concat", False),
    ([100, 1, 256, 63, 0, 130], 4, 2, 128, 4, "concat", True),
    ([129, 40, 300], 2, 2, 64, 4, "concat", True),
])
def test_packed_form_matches_padded_form(lens, HQ, H, D, M, score, decay, monkeypatch):
    """The tensor-core packed-document form against the padded batch on the same bf16 inputs: the
    same function, so outputs and gradients agree to the bf16 tolerance; the packed form must be
    the one AUTO takes for these inputs."""
    import linatt_b200.varlen as vl

    T = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32).cuda()
    g = torch.Generator().manual_seed(T)
    q = (torch.randn(1, T, HQ, D, generator=g) / D ** 0.5).bfloat16().cuda()
    k = F.normalize(torch.randn(1, T, H, D, generator=g), dim=-1).bfloat16().cuda()
    v = torch.randn(1, T, H, D, generator=g).bfloat16().cuda()
    do = torch.randn(1, T, HQ, D, generator=g).bfloat16().cuda()
    c = -F.softplus(torch.randn(1, T, HQ, generator=g)).cumsum(1).cuda() if decay else None
    assert vl._packed_ok(q, k, v, M, score, c, len(lens))

    def run(packed):
        monkeypatch.setattr(vl, "_packed_ok", (lambda *a: True) if packed else (lambda *a: False))
        leaves = [x.clone().requires_grad_(True) for x in (q, k, v)] + ([c.clone().requires_grad_(True)] if decay else [])
        o = vl.parallel_kata_attn_varlen(*leaves[:3], cu, num_groups=M, score=score, max_seqlen=max(lens),
                                         c=leaves[3] if decay else None)
        o.backward(do)
        torch.cuda.synchronize()
        return [o.detach()] + [x.grad for x in leaves]

    got, ref = run(True), run(False)
    for name, a, b in zip(("o", "dq", "dk", "dv", "dc"), got, ref):
        assert torch.isfinite(a.float()).all(), name
        assert _rel(a, b) < 1e-2, name
