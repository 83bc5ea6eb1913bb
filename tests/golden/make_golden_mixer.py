"""Generate the golden fixtures of the KATA mixer (prologue, attention, epilogue) from the reference.

Run where the reference checkout is importable (never needed at test time):

    LINATT_REFERENCE=/path/to/linatt python tests/golden/make_golden_mixer.py

It builds the reference's own ``KataAttention`` (kata/layer.py:45-292) and runs its ``forward``
(:286-541) and autograd backward on CPU in float64.  The fla kernels that layer calls are GPU-only
(Triton), so each is replaced by the pure-PyTorch statement of the same operation:

* ``ShortConvolution`` (an ``nn.Conv1d`` subclass) -> ``F.conv1d`` with its own weight, causal
  padding K - 1, SiLU (the definition fla's kernels implement);
* ``RMSNorm`` -> fla's own ``fla.modules.layernorm.rms_norm_ref``;
* ``l2norm`` -> x / sqrt(sum x^2 + 1e-6) (fla ``l2norm_fwd_kernel``, fla/modules/l2norm.py:42);
* ``RotaryEmbedding`` -> fla's own ``fla.modules.rotary.rotary_embedding_ref`` with the cos / sin
  tables built as fla builds them (fp32 angles, cast to the activations' dtype);
* the attention op -> the reference's own ``_kata_decay_ref`` (kata/parallel_kata_attn.py:291),
  with c = 0 for the undecayed forms.

Stored per case (float32, ``tests/golden/mixer_golden.npz``): the input x, every parameter of
the layer (reference names), the upstream gradient, the output and the gradients of x and of every
parameter.
"""

from __future__ import annotations

import math
import os
import sys
from pathlib import Path

import numpy as np

REF = os.environ.get("LINATT_REFERENCE")
if not REF:
    sys.exit("set LINATT_REFERENCE to the reference checkout")
sys.path.insert(0, REF)

import torch  # noqa: E402
import torch.nn as nn  # noqa: E402
import torch.nn.functional as F  # noqa: E402
from fla.modules.layernorm import rms_norm_ref  # noqa: E402
from fla.modules.rotary import rotary_embedding_ref  # noqa: E402

import kata.layer as KL  # noqa: E402
from kata.parallel_kata_attn import _kata_decay_ref  # noqa: E402


class _Conv(nn.Conv1d):
    def __init__(self, hidden_size, kernel_size, bias=False, activation="silu", **kw):
        super().__init__(hidden_size, hidden_size, kernel_size, groups=hidden_size, bias=bias,
                         padding=kernel_size - 1)
        self.act = activation

    def forward(self, x, cache=None, output_final_state=False, **kw):
        T = x.shape[1]
        y = F.conv1d(x.transpose(1, 2), self.weight, self.bias, padding=self.kernel_size[0] - 1,
                     groups=x.shape[-1])[..., :T].transpose(1, 2)
        return (F.silu(y) if self.act else y), None


class _RMS(nn.Module):
    def __init__(self, hidden_size, elementwise_affine=True, eps=1e-5, dtype=None, **kw):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size, dtype=dtype)) if elementwise_affine else None

    def forward(self, x):
        w = self.weight if self.weight is not None else torch.ones(x.shape[-1], dtype=x.dtype)
        return rms_norm_ref(x, w.to(x.dtype), None, eps=self.eps)


class _Rot(nn.Module):
    def __init__(self, dim, base=10000.0, interleaved=False, **kw):
        super().__init__()
        self.dim, self.base, self.interleaved = dim, float(base), interleaved

    def forward(self, q, k, seqlen_offset=0, max_seqlen=None, **kw):
        T = q.shape[1]
        inv = 1.0 / (self.base ** (torch.arange(0, self.dim, 2, dtype=torch.float32) / self.dim))
        fr = torch.outer(torch.arange(max(T, max_seqlen or 0), dtype=torch.float32), inv)
        cos, sin = torch.cos(fr).to(q.dtype)[:T], torch.sin(fr).to(q.dtype)[:T]
        return rotary_embedding_ref(q, cos, sin, self.interleaved), rotary_embedding_ref(k, cos, sin, self.interleaved)


def _attn(q, k, v, num_groups=4, scale=None):
    s = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1] // num_groups)
    c = torch.zeros(q.shape[0], q.shape[1], q.shape[2], dtype=q.dtype)
    return _kata_decay_ref(q, k, v, c, num_groups, s)


def _attn_decay(q, k, v, c, num_groups=2, scale=None):
    s = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1] // num_groups)
    return _kata_decay_ref(q, k, v, c.to(q.dtype), num_groups, s)


KL.ShortConvolution = _Conv
KL.RMSNorm = _RMS
KL.RotaryEmbedding = _Rot
KL.l2norm = lambda x: x * torch.rsqrt(x.pow(2).sum(-1, keepdim=True) + 1e-6)
KL.parallel_kata_attn = _attn
KL.parallel_kata_attn_decay = _attn_decay

# name -> (constructor kwargs, B, T)
CASES = {
    "conv_m4": (dict(hidden_size=128, num_heads=2, spd_num_groups=4, use_short_conv=True, norm_eps=1e-6), 2, 40),
    "l2_rope_m2": (dict(hidden_size=128, num_heads=2, spd_num_groups=2, use_short_conv=True, qk_norm=True,
                        norm_q="l2", norm_k="l2", use_rope=True), 2, 37),
    "rms_ropegroup_m4": (dict(hidden_size=128, num_heads=2, spd_num_groups=4, qk_norm=True, norm_q="rmsnorm",
                              norm_k="rmsnorm", use_rope=True, rope_group=True), 1, 50),
    "decay_conv_m2": (dict(hidden_size=128, num_heads=2, spd_num_groups=2, use_short_conv=True, use_decay=True), 2,
                      33),
    "offset_m4": (dict(hidden_size=128, num_heads=2, spd_num_groups=4, use_offset_gate=True), 1, 45),
    "gqa_conv_m4": (dict(hidden_size=128, num_heads=4, num_kv_heads=2, spd_num_groups=4, use_short_conv=True,
                         expand_k=2.0, expand_v=2.0), 1, 30),
}


def main() -> None:
    out = {}
    for name, (kw, B, T) in CASES.items():
        torch.manual_seed(hash(name) % 1000)
        layer = KL.KataAttention(feature_map="kata_quadratic", mode="chunk", **kw).double()
        with torch.no_grad():  # non-trivial norm scales, so their gradients are exercised too
            for pn, p in layer.named_parameters():
                if pn.endswith("norm.weight"):
                    p.add_(0.1 * torch.randn_like(p))
        x = torch.randn(B, T, kw["hidden_size"], dtype=torch.float64, requires_grad=True)
        o, _, _ = layer(x)
        do = torch.randn_like(o)
        o.backward(do)
        out[f"{name}/x"] = x.detach().float().numpy()
        out[f"{name}/do"] = do.float().numpy()
        out[f"{name}/o"] = o.detach().float().numpy()
        out[f"{name}/dx"] = x.grad.float().numpy()
        for pn, p in layer.named_parameters():
            out[f"{name}/p/{pn}"] = p.detach().float().numpy()
            out[f"{name}/g/{pn}"] = p.grad.float().numpy()
        print(name, o.shape, [pn for pn, _ in layer.named_parameters()])
    dst = Path(__file__).with_name("mixer_golden.npz")
    np.savez_compressed(dst, **out)
    print("wrote", dst, sum(v.nbytes for v in out.values()) // 1024, "KiB")


if __name__ == "__main__":
    main()
