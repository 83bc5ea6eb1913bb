"""Golden fixtures for the SPD delta rule (``kata/spd/flash_delta.py``), generated from the
reference's own code in a container where the reference checkout is importable:

    LINATT_REFERENCE=/path/to/linatt python tests/golden/make_golden_delta.py

The reference kernels are Triton; they are run under the Triton CPU interpreter
(``TRITON_INTERPRET=1``) with fp32 inputs, calling each autotuned kernel's underlying JIT function
(the autotuner needs a GPU driver).  The interpreter computes ``tl.dot`` on bf16 operands
incorrectly, and every inter-chunk product and the readout of ``flash_delta`` cast to bf16
(kata/spd/flash_delta.py:110-111, :964-967), so the only part that runs faithfully is the
pseudo-value solve U of a single chunk (K14, ``flash_delta_U``, :186-212), whose dots are fp32.
These fixtures therefore pin U = (I + diag(beta) tril(A_kk,-1))^{-1} diag(beta) V and the
kernel/scale conventions at T = C = 64; the readout and the backward are pinned by construction
in ``oracle/delta_oracle.py``.  Stored as float32 in ``tests/golden/delta_golden.npz``.
"""

from __future__ import annotations

import importlib
import os
import sys
from pathlib import Path

import numpy as np

os.environ["TRITON_INTERPRET"] = "1"
REF = os.environ.get("LINATT_REFERENCE")
if not REF:
    sys.exit("set LINATT_REFERENCE to the reference checkout")
sys.path.insert(0, REF)

import torch  # noqa: E402
from triton.runtime.autotuner import Autotuner  # noqa: E402

fdm = importlib.import_module("kata.spd.flash_delta")
for _name in dir(fdm):
    _obj = getattr(fdm, _name)
    if isinstance(_obj, Autotuner):
        setattr(fdm, _name, _obj.fn)

OUT = Path(__file__).resolve().parent / "delta_golden.npz"

# (name, B, T, H, D, Dv, M, scale)
CASES = [
    ("m1", 1, 64, 2, 32, 32, 1, 0.5),
    ("m2", 1, 64, 2, 32, 32, 2, 0.5),
    ("m4_default_scale", 1, 64, 1, 64, 64, 4, None),
]


def main():
    out = {}
    for i, (name, B, T, H, D, Dv, M, scale) in enumerate(CASES):
        g = torch.Generator().manual_seed(2000 + i)
        q = torch.randn(B, T, H, D, generator=g)
        k = torch.randn(B, T, H, D, generator=g)
        k = k / k.norm(dim=-1, keepdim=True)
        v = torch.randn(B, T, H, Dv, generator=g)
        beta = torch.sigmoid(torch.randn(B, T, H, generator=g))
        U = fdm.flash_delta_U(q, k, v, beta, M, scale=scale, C=64)
        for key, val in dict(q=q, k=k, v=v, beta=beta, U=U).items():
            out[f"{name}/{key}"] = val.float().numpy()
        out[f"{name}/meta"] = np.array([B, T, H, D, Dv, M, -1.0 if scale is None else scale], dtype=np.float64)
        print(name, "done", flush=True)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1e6:.2f} MB)")


if __name__ == "__main__":
    main()
