"""Same-box bar: the reference's own Triton kernels timed on this GPU beside this library's kernels.

MEASUREMENT / TEST INFRASTRUCTURE ONLY: nothing in ``linatt_b200`` imports this file, and the
reference code it runs is never part of the product path.

The reference checkout is given on the command line (``--reference-root``; it is not part of this
repository).  Its modules are imported by file path under the package name ``kata`` without
running ``kata/__init__.py`` (which pulls in model code); Triton JIT-compiles them for this GPU and
autotunes them at their first call, outside the timed region.

Workloads (seeded synthetic inputs with the benchmark shapes):
  attn   config 3: B=16, T=4096, H=8, D=Dv=128, M=4 concat, bf16, q,k,v ~ N(0,1)/sqrt(128).
         Reference: forward kernel K1 (kata/kernels/parallel_kata.py:10-197), launched with the
         arguments of parallel_kata_attn_fwd_impl (kata/parallel_kata_attn.py:265-287) plus the
         VARLEN=False constexpr that launcher omits at HEAD, and the backward dispatcher
         parallel_kata_attn_bwd_triton (kata/parallel_kata_attn.py:364-529: delta preprocess,
         dq_M4, dkdv_M4), unmodified.  Ours: kata_attn_fwd, kata_attn_bwd phases 1 (dq) and 2 (dk/dv).
  gdn    config 2: fla's chunk_gated_delta_rule (fla/ops/gated_delta_rule/chunk.py:365, Triton;
         third-party, installed) forward + backward at B=8, T=2048, H=12, K=V=64, bf16 inputs,
         against linatt_b200.gated_delta_rule.chunk_gated_delta_rule.  fla 0.5.1 dispatches some
         backward pieces to an optional TileLang backend when tilelang is importable; on B200 that
         backend's chunk_bwd_dqkwg raised a misaligned-address fault, so this script sets
         FLA_DISABLE_BACKEND_DISPATCH=1 (fla's own switch) and times fla's default Triton kernels.
  delta  the SPD delta rule at the 200M mixer geometry (B=8, T=2048, H=12, D=Dv=64, M=4, scale 0.5,
         normalised, bf16 inputs): the reference's flash_delta (kata/spd/flash_delta.py:1111)
         forward + backward against linatt_b200.spd.flash_delta.
Each pass: median CUDA-event time over --reps calls after warm-up (inputs above L2 for attn; the
others rotate 4 input sets).  Also the relative L2 distance between the two implementations'
outputs and gradients.  Prints one JSON object.

Usage: python oracle/triton_bar.py --reference-root PATH [--what attn,gdn,delta] [--reps N]
"""

from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import statistics
import sys
import types
from pathlib import Path

import torch
import torch.nn.functional as F

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def load_reference(root: Path):
    """Register ``kata`` / ``kata.spd`` as namespace stubs over the checkout and import the modules
    on the hot path (their own imports are torch, triton and kata.kernels.*)."""
    for name, sub in (("kata", "kata"), ("kata.spd", "kata/spd")):
        m = types.ModuleType(name)
        m.__path__ = [str(root / sub)]
        sys.modules[name] = m
    pka = importlib.import_module("kata.parallel_kata_attn")
    kern = importlib.import_module("kata.kernels.parallel_kata")
    fd = importlib.import_module("kata.spd.flash_delta")
    return pka, kern, fd


def rel(a, b) -> float:
    a, b = a.double(), b.double()
    n = b.norm()
    return float((a - b).norm() / n) if n > 0 else float((a - b).norm())


def time_ms(fn, reps: int, warm: int = 3) -> float:
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(reps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        out.append(s.elapsed_time(e))
    return statistics.median(out)


# ------------------------------------------------------------------------------------------------
def bar_attn(ref, reps: int) -> dict:
    import triton

    from linatt_b200 import _lib

    rpka, kern, _ = ref
    B, T, H, D, M = 16, 4096, 8, 128, 4
    scale = 1.0 / math.sqrt(D // M)
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    q, k, v = ((torch.randn(B, T, H, D, device=dev, generator=g) / math.sqrt(D)).bfloat16() for _ in range(3))
    do = torch.randn(B, T, H, D, device=dev, generator=g).bfloat16()

    def ref_fwd():
        o = torch.empty_like(v)
        den = torch.empty(B, T, H, device=dev, dtype=torch.float32)
        grid = lambda meta: (1, triton.cdiv(T, meta["bT"]), B * H)  # noqa: E731
        kern.parallel_kata_attn_fwd_kernel[grid](q, k, v, o, den, den, scale, T, H=H, M=M, d_k=D, d_v=D, HQ=H, G=1,
                                                 bV=D, HAS_DECAY=False, VARLEN=False)
        return o, den

    r_o, r_den = ref_fwd()
    ref_bwd = lambda: rpka.parallel_kata_attn_bwd_triton(q, k, v, r_o, r_den, do, M, scale)  # noqa: E731
    r_dq, r_dk, r_dv = ref_bwd()
    t_ref_fwd = time_ms(ref_fwd, reps)
    t_ref_bwd = time_ms(ref_bwd, reps)

    L = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    o = torch.empty_like(v)
    den = torch.empty(B, T, H, device=dev)
    fa = _lib.AttnFwdArgs(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), o=o.data_ptr(), den=den.data_ptr(),
                          dtype=1, B=B, T=T, H=H, HQ=H, D=D, Dv=D, M=M, score=0, algo=1, scale=scale)
    our_fwd = lambda: _lib.check(L.kata_attn_fwd(fa, st), "kata_attn_fwd")  # noqa: E731
    our_fwd()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    ba = _lib.AttnBwdArgs(q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), o=o.data_ptr(), den=den.data_ptr(),
                          dout=do.data_ptr(), dq=dq.data_ptr(), dk=dk.data_ptr(), dv=dv.data_ptr(), dtype=1, B=B, T=T,
                          H=H, HQ=H, D=D, Dv=D, M=M, score=0, algo=1, scale=scale)
    nb = L.kata_attn_bwd_workspace_bytes(ba)
    ws = torch.empty(nb, dtype=torch.uint8, device=dev)
    ba.workspace, ba.workspace_bytes = ws.data_ptr(), nb

    def our_pass(ph):
        ba.phases = ph
        _lib.check(L.kata_attn_bwd(ba, st), "kata_attn_bwd")

    our_pass(0)
    torch.cuda.synchronize()
    t_fwd = time_ms(our_fwd, reps)
    t_dq = time_ms(lambda: our_pass(1), reps)
    t_dkdv = time_ms(lambda: our_pass(2), reps)
    t_bwd = time_ms(lambda: our_pass(0), reps)
    flops = 3.5 * B * H * 2.0 * (T * (T + 1) / 2) * (2 * D + 2 * D)
    return {
        "workload": "KATA-SPD attention fwd+bwd, config 3 (B16 T4096 H8 D128, M=4 concat, bf16)",
        "reference_triton_ms": {"fwd": t_ref_fwd, "bwd": t_ref_bwd, "step": t_ref_fwd + t_ref_bwd},
        "ours_ms": {"fwd": t_fwd, "bwd_dq": t_dq, "bwd_dkdv": t_dkdv, "bwd": t_bwd, "step": t_fwd + t_bwd},
        "speedup": {"fwd": t_ref_fwd / t_fwd, "bwd": t_ref_bwd / t_bwd,
                    "step": (t_ref_fwd + t_ref_bwd) / (t_fwd + t_bwd)},
        "tflops": {"reference": flops / ((t_ref_fwd + t_ref_bwd) / 1e3) / 1e12,
                   "ours": flops / ((t_fwd + t_bwd) / 1e3) / 1e12},
        "rel_l2_ours_vs_reference": {"o": rel(o, r_o), "den": rel(den, r_den), "dq": rel(dq, r_dq),
                                     "dk": rel(dk, r_dk), "dv": rel(dv, r_dv)},
    }


# ------------------------------------------------------------------------------------------------
def _gdn_inputs(dev, n):
    Bg, Tg, Hg, Kg = 8, 2048, 12, 64
    g = torch.Generator(device=dev).manual_seed(99)
    sets = []
    for _ in range(n):
        q = torch.randn(Bg, Tg, Hg, Kg, device=dev, generator=g).bfloat16()
        k = F.normalize(torch.randn(Bg, Tg, Hg, Kg, device=dev, generator=g), dim=-1).bfloat16()
        v = torch.randn(Bg, Tg, Hg, Kg, device=dev, generator=g).bfloat16()
        beta = torch.sigmoid(torch.randn(Bg, Tg, Hg, device=dev, generator=g))
        gate = -F.softplus(torch.randn(Bg, Tg, Hg, device=dev, generator=g))
        do = torch.randn(Bg, Tg, Hg, Kg, device=dev, generator=g).bfloat16()
        sets.append((q, k, v, gate, beta, do))
    return sets


def _fwd_bwd(fn, args, do):
    leaves = [x.detach().clone().requires_grad_(True) for x in args]
    o = fn(*leaves)
    o = o[0] if isinstance(o, tuple) else o
    o.backward(do)
    return [o.detach()] + [x.grad for x in leaves]


def bar_gdn(reps: int) -> dict:
    from fla.ops.gated_delta_rule import chunk_gated_delta_rule as fla_gdn

    from linatt_b200.gated_delta_rule import chunk_gated_delta_rule as our_gdn

    dev = torch.device("cuda")
    sets = _gdn_inputs(dev, 4)
    it = {"i": 0}

    def step(fn):
        def run():
            q, k, v, gate, beta, do = sets[it["i"] % 4]
            it["i"] += 1
            _fwd_bwd(fn, (q, k, v, gate, beta), do)
        return run

    q, k, v, gate, beta, do = sets[0]
    a = _fwd_bwd(fla_gdn, (q, k, v, gate, beta), do)
    b = _fwd_bwd(our_gdn, (q, k, v, gate, beta), do)
    names = ["o", "dq", "dk", "dv", "dg", "dbeta"]
    t_fla = time_ms(step(fla_gdn), reps)
    t_our = time_ms(step(our_gdn), reps)
    return {"workload": "chunk_gated_delta_rule fwd+bwd, config 2 (B8 T2048 H12 K=V=64, bf16)",
            "fla_triton_ms": t_fla, "ours_ms": t_our, "speedup": t_fla / t_our,
            "rel_l2_ours_vs_fla": {n: rel(y.float(), x.float()) for n, x, y in zip(names, a, b)}}


def bar_delta(ref, reps: int) -> dict:
    from linatt_b200.spd import flash_delta as our_fd

    _, _, fd = ref
    dev = torch.device("cuda")
    Bd, Td, Hd, Dd, Md = 8, 2048, 12, 64, 4
    g = torch.Generator(device=dev).manual_seed(77)
    sets = []
    for _ in range(4):
        q = F.normalize(torch.randn(Bd, Td, Hd, Dd, device=dev, generator=g), dim=-1).bfloat16()
        k = F.normalize(torch.randn(Bd, Td, Hd, Dd, device=dev, generator=g), dim=-1).bfloat16()
        v = torch.randn(Bd, Td, Hd, Dd, device=dev, generator=g).bfloat16()
        beta = torch.sigmoid(torch.randn(Bd, Td, Hd, device=dev, generator=g)).bfloat16()
        do = torch.randn(Bd, Td, Hd, Dd, device=dev, generator=g)
        sets.append((q, k, v, beta, do))
    ref_fn = lambda q, k, v, b: fd.flash_delta(q, k, v, b, Md, scale=0.5, normalize=True)  # noqa: E731
    our_fn = lambda q, k, v, b: our_fd(q, k, v, b, Md, scale=0.5, normalize=True)  # noqa: E731
    it = {"i": 0}

    def step(fn):
        def run():
            q, k, v, beta, do = sets[it["i"] % 4]
            it["i"] += 1
            _fwd_bwd(fn, (q, k, v, beta), do)
        return run

    q, k, v, beta, do = sets[0]
    a = _fwd_bwd(ref_fn, (q, k, v, beta), do)
    b = _fwd_bwd(our_fn, (q, k, v, beta), do)
    t_ref = time_ms(step(ref_fn), reps)
    t_our = time_ms(step(our_fn), reps)
    return {"workload": "flash_delta fwd+bwd, B8 T2048 H12 D=Dv=64, M=4, scale 0.5, normalised, bf16",
            "reference_triton_ms": t_ref, "ours_ms": t_our, "speedup": t_ref / t_our,
            "rel_l2_ours_vs_reference": {n: rel(y.float(), x.float())
                                         for n, x, y in zip(["o", "dq", "dk", "dv", "dbeta"], a, b)}}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference-root", type=Path, required=True)
    ap.add_argument("--what", default="attn,gdn,delta")
    ap.add_argument("--reps", type=int, default=20)
    a = ap.parse_args()
    os.environ["FLA_DISABLE_BACKEND_DISPATCH"] = "1"  # fla's Triton kernels, not its TileLang backend
    ref = load_reference(a.reference_root.resolve())
    torch.cuda.init()
    out = {"gpu": torch.cuda.get_device_name(0)}
    import triton

    out["triton"] = triton.__version__
    for w in a.what.split(","):
        if w == "attn":
            out["attn"] = bar_attn(ref, a.reps)
        elif w == "gdn":
            out["gdn"] = bar_gdn(a.reps)
        elif w == "delta":
            out["delta"] = bar_delta(ref, a.reps)
        print(json.dumps({w: out[w]}), flush=True)
    print(json.dumps(out))


if __name__ == "__main__":
    main()
