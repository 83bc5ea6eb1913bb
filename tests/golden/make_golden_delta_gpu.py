"""Golden fixtures for the whole SPD delta rule, made by the reference's own Triton kernels on a GPU.

    python tests/golden/make_golden_delta_gpu.py --reference-root PATH [--what delta,spd] [--out-dir DIR]

The CPU interpreter cannot run the reference's bf16 tensor-core dots (its bf16 ``tl.dot`` is wrong
in this image), so ``make_golden_delta.py`` pins only the single-chunk pseudo-value solve.  This
script runs ``kata/spd/flash_delta.py`` compiled by Triton for the GPU it runs on (a B200 here) and
stores, per case, the inputs and the reference's outputs:

  * U    = flash_delta_U                (K14, kata/spd/flash_delta.py:186-212), multi-chunk
  * num  = flash_delta_readout(U)       (K15, :975-985)
  * den  = flash_delta_den              (K16, :1049-1057)
  * o, dq, dk, dv, dbeta = flash_delta forward and backward through _FlashDelta (:1060-1116),
    for normalize True and False (dq, dk, dv, dbeta in the input dtype, as the reference returns)

Inputs follow the layer (kata/layer.py:399-418): q, k, v, beta cast to bf16, T a multiple of 64;
q, k L2-normalised per head, beta = sigmoid(N(0,1)); dO ~ N(0,1) fp32.  Every tensor is stored as
float32 (bf16 values are exact in it) in ``tests/golden/delta_golden_gpu.npz``.

``--what spd`` adds the head-major sibling ``spd_chunk_scan`` (kata/spd/chunk_scan.py:295-406, sum
mode: o, den), run by the reference's own Triton kernels on the same kind of inputs (bf16,
head-major (B, H, T, D)), into ``tests/golden/spd_golden_gpu.npz``.  ``spd_state_lin``
(chunk_state_lin.py) and ``flash_delta_state`` (chunk_state_v2.py) have launch helpers here as well
(each works around a launcher bug at HEAD), but their kernels do not fit on a B200 (see SPD_CASES).

The reference checkout is given on the command line and is imported by file path; it is not part
of this repository.
"""

from __future__ import annotations

import argparse
import importlib
import sys
import types
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent

# (name, B, T, H, D, Dv, M, scale, normalize)
CASES = [
    ("m4_norm", 1, 256, 2, 64, 64, 4, 0.5, True),
    ("m4_raw", 1, 192, 2, 64, 64, 4, 0.5, False),
    ("m2_norm_default_scale", 2, 128, 1, 32, 32, 2, None, True),
    ("m1_raw", 1, 256, 1, 32, 32, 1, 0.5, False),
]


# (name, function, B, H, T, D, Dv, M, scale)
# spd_state_lin's and flash_delta_state's own Triton kernels do not fit on a B200: compiled for
# sm_100 they ask for 608-736 of the SM's 512 tensor-memory columns and Triton refuses to launch
# them (OutOfResources).  Their functions are pinned through flash_delta instead (the readout
# numerator tril(kappa(q,k)) U, and the raw-numerator delta rule); the launch helpers below are kept
# for a GPU where they fit.
SPD_CASES = [
    ("scan_m4", "chunk_scan", 1, 2, 256, 64, 64, 4, 0.5),
    ("scan_m2_default_scale", "chunk_scan", 2, 1, 128, 32, 32, 2, None),
]


def load_reference(root: Path, module: str):
    for name, sub in (("kata", "kata"), ("kata.spd", "kata/spd")):
        if name not in sys.modules:
            m = types.ModuleType(name)
            m.__path__ = [str(root / sub)]
            sys.modules[name] = m
    return importlib.import_module(f"kata.spd.{module}")


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference-root", type=Path, required=True)
    ap.add_argument("--what", default="delta,spd")
    ap.add_argument("--out-dir", type=Path, default=HERE)
    a = ap.parse_args()
    root = a.reference_root.resolve()
    dev = torch.device("cuda")
    jobs = []
    if "delta" in a.what.split(","):
        fd = load_reference(root, "flash_delta")
        jobs.append(("delta_golden_gpu.npz", [(lambda i=i, c=c, o=None: run_case(fd, dev, i, c, o), c[0])
                                               for i, c in enumerate(CASES)]))
    if "spd" in a.what.split(","):
        mods = {"state_lin": load_reference(root, "chunk_state_lin"), "chunk_scan": load_reference(root, "chunk_scan"),
                "delta_state": load_reference(root, "chunk_state_v2")}
        jobs.append(("spd_golden_gpu.npz", [(lambda i=i, c=c, o=None: run_spd_case(mods, dev, i, c, o), c[0])
                                             for i, c in enumerate(SPD_CASES)]))
    for fname, cases in jobs:
        out = {}
        for fn, name in cases:
            try:
                fn(o=out)
            except Exception as e:  # noqa: BLE001 -- report and keep the other cases
                print(name, "FAILED", type(e).__name__, str(e)[:300], flush=True)
        out["gpu"] = np.array(torch.cuda.get_device_name(0))
        path = a.out_dir / fname
        np.savez_compressed(path, **out)
        print(f"wrote {path} ({path.stat().st_size / 1e6:.2f} MB)")


def state_lin_reference(m, q, k, v, do, M, scale):
    """spd_state_lin forward and backward.  Its forward kernel's autotuner names a reset_to_zero
    argument "S" that the kernel does not have (kata/spd/chunk_state_lin.py:22-23 vs :26-33), so at
    HEAD _StateLin.forward raises KeyError; the forward kernel is launched here through its JIT
    function with one of its own configs (num_warps=4, num_stages=1) on a zeroed state.  Its
    backward launcher passes H= to both backward kernels, whose signatures have no H (:465-484 vs
    :166-184, :308-325), so they are launched with _StateLin.backward's other arguments."""
    B, H, T, D = q.shape
    DV = v.shape[-1]
    E, E2, BI = m._lin_params(D, M, None)
    scale = 1.0 / E if scale is None else scale
    ss = scale ** 0.5
    q, k, v = (x.contiguous() for x in (q, k, v))
    f32 = dict(device=q.device, dtype=torch.float32)
    o = torch.empty(B, H, T, DV, **f32)
    S = torch.zeros(B * H, E2, DV, **f32)
    m._state_lin_kernel.fn[(B * H,)](q, k, v, o, S, ss, T, D=D, E=E, M=M, DV=DV, C=64, E2=E2, BI=BI, num_warps=4,
                                      num_stages=1)
    do = do.contiguous()
    dq, dk1, dv1, dk2, dv2 = (torch.empty_like(x) for x in (q, k, v, k, v))
    Hst = torch.zeros(B * H, E2, DV, **f32)
    Rst = torch.zeros(B * H, E2, DV, **f32)
    m._lin_bwd_p1_kernel[(B * H,)](q, k, v, do, dq, dk1, dv1, Hst, ss, T, D=D, E=E, M=M, DV=DV, C=64, E2=E2, BI=BI)
    m._lin_bwd_p2_kernel[(B * H,)](q, k, v, do, dk2, dv2, Rst, ss, T, D=D, E=E, M=M, DV=DV, C=64, E2=E2, BI=BI)
    return o, dq, dk1 + dk2, dv1 + dv2


def delta_state_forward(m, q, k, v, beta, M, scale):
    """flash_delta_state's forward, (o, U, S).  Its launcher spd_delta_state_v2 passes H= to
    _state_v2_kernel, whose signature has no H (kata/spd/chunk_state_v2.py:340 vs :372-390), so at
    HEAD it raises; this replicates that launcher's tile choices and launch without the H argument."""
    B, H, T, D = q.shape
    DV = v.shape[-1]
    E = D // M
    scale = 1.0 / E if scale is None else scale
    DVB = DV
    BI = max(1, 256 // E)
    while E % BI != 0:
        BI //= 2
    o = torch.empty(B, H, T, DV, device=q.device, dtype=torch.float32)
    S = torch.zeros(B * H, E * E, DV, device=q.device, dtype=torch.float32)
    U = torch.empty(B, H, T, DV, device=q.device, dtype=torch.float32)
    m._state_v2_kernel[(B * H,)](q.contiguous(), k.contiguous(), v.contiguous(), beta.contiguous(), o, U, S,
                                 scale ** 0.5, T, D=D, E=E, M=M, DV=DV, DVB=DVB, C=64, E2=E * E, BI=BI, WRITE_U=True)
    return o, U, S


def run_spd_case(mods, dev, i, case, out):
    name, fn, B, H, T, D, Dv, M, scale = case
    g = torch.Generator().manual_seed(4000 + i)
    q = F.normalize(torch.randn(B, H, T, D, generator=g), dim=-1).bfloat16().to(dev)
    k = F.normalize(torch.randn(B, H, T, D, generator=g), dim=-1).bfloat16().to(dev)
    v = torch.randn(B, H, T, Dv, generator=g).bfloat16().to(dev)
    beta = torch.sigmoid(torch.randn(B, H, T, generator=g)).bfloat16().to(dev)
    do = torch.randn(B, H, T, Dv, generator=g).to(dev)
    tensors = dict(q=q, k=k, v=v, beta=beta, do=do)
    if fn == "chunk_scan":
        o, den = mods["chunk_scan"].spd_chunk_scan(q, k, v, M, "sum", scale=scale)
        tensors.update(o=o, den=den)
    else:
        leaves = [x.clone().requires_grad_(True) for x in ((q, k, v) if fn == "state_lin" else (q, k, v, beta))]
        if fn == "state_lin":
            o, dq, dk, dv = state_lin_reference(mods["state_lin"], q, k, v, do, M, scale)
            tensors.update(o=o, dq=dq, dk=dk, dv=dv)
        else:
            m = mods["delta_state"]
            o, U, S = delta_state_forward(m, q, k, v, beta, M, scale)
            dq, dk, dv, db = m.spd_delta_state_bwd(q, k, v, beta, do, U, S, M, scale=scale, C=64)
            tensors.update(o=o, dq=dq, dk=dk, dv=dv, dbeta=db)
    torch.cuda.synchronize()
    for key, val in tensors.items():
        out[f"{name}/{key}"] = val.float().cpu().numpy()
    out[f"{name}/meta"] = np.array([B, H, T, D, Dv, M, -1.0 if scale is None else scale], dtype=np.float64)
    out[f"{name}/fn"] = np.array(fn)
    print(name, "done", {k_: float(v_.float().norm()) for k_, v_ in tensors.items()}, flush=True)


def run_case(fd, dev, i, case, out):
    name, B, T, H, D, Dv, M, scale, normalize = case
    g = torch.Generator().manual_seed(3000 + i)
    q = F.normalize(torch.randn(B, T, H, D, generator=g), dim=-1).bfloat16().to(dev)
    k = F.normalize(torch.randn(B, T, H, D, generator=g), dim=-1).bfloat16().to(dev)
    v = torch.randn(B, T, H, Dv, generator=g).bfloat16().to(dev)
    beta = torch.sigmoid(torch.randn(B, T, H, generator=g)).bfloat16().to(dev)
    do = torch.randn(B, T, H, Dv, generator=g).to(dev)
    U = fd.flash_delta_U(q, k, v, beta, M, scale=scale, C=64)
    num = fd.flash_delta_readout(q, k, U, M, scale=scale, C=64)
    den = fd.flash_delta_den(q, k, M, scale=scale, C=64)
    leaves = [x.clone().requires_grad_(True) for x in (q, k, v, beta)]
    o = fd.flash_delta(*leaves, M, scale=scale, C=64, normalize=normalize)
    o.backward(do)
    torch.cuda.synchronize()
    tensors = dict(q=q, k=k, v=v, beta=beta, do=do, U=U, num=num, den=den, o=o.detach(),
                   dq=leaves[0].grad, dk=leaves[1].grad, dv=leaves[2].grad, dbeta=leaves[3].grad)
    for key, val in tensors.items():
        out[f"{name}/{key}"] = val.float().cpu().numpy()
    out[f"{name}/meta"] = np.array([B, T, H, D, Dv, M, -1.0 if scale is None else scale, float(normalize)],
                                   dtype=np.float64)
    print(name, "done", {k_: float(v_.float().norm()) for k_, v_ in tensors.items()}, flush=True)


if __name__ == "__main__":
    main()
