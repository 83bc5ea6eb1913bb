"""The C-ABI library builds, loads, exports every symbol declared in include/*.h, and rejects bad
arguments on the host (these paths never touch a GPU)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    syms = set()
    for h in (ROOT / "include").glob("*.h"):
        for m in re.finditer(r"KATA_API\s+[\w\s\*]+?\b(kata_\w+)\s*\(", h.read_text()):
            syms.add(m.group(1))
    return sorted(syms)


@pytest.fixture(scope="module")
def L():
    from linatt_b200 import build, _lib

    build.build()
    return _lib.lib()


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("kata_attn_fwd", "kata_attn_bwd", "kata_attn_bwd_workspace_bytes", "kata_strerror",
              "kata_abi_version"):
        assert s in syms


def test_library_exports_every_declared_symbol(L):
    for s in declared_symbols():
        assert hasattr(L, s), f"{s} not exported"


def test_abi_version_and_strerror(L):
    from linatt_b200 import _lib

    assert L.kata_abi_version() == _lib.ABI_VERSION
    assert L.kata_strerror(0) == b"ok"
    assert b"workspace" in L.kata_strerror(-5)
    assert L.kata_strerror(12345) == b"unknown error"


def test_host_side_validation(L):
    from linatt_b200 import _lib

    assert L.kata_attn_fwd(None, None) == -1
    a = _lib.AttnFwdArgs(dtype=7, B=1, T=8, H=1, HQ=1, D=64, Dv=64, M=4, score=0, algo=0, scale=1.0)
    assert L.kata_attn_fwd(a, None) == -2  # dtype
    a = _lib.AttnFwdArgs(dtype=1, B=1, T=8, H=2, HQ=3, D=64, Dv=64, M=4, score=0, algo=0, scale=1.0)
    assert L.kata_attn_fwd(a, None) == -3  # HQ % H
    a = _lib.AttnFwdArgs(dtype=1, B=1, T=8, H=1, HQ=1, D=64, Dv=64, M=3, score=0, algo=0, scale=1.0)
    assert L.kata_attn_fwd(a, None) == -3  # D % M
    a = _lib.AttnFwdArgs(dtype=1, B=1, T=8, H=1, HQ=1, D=64, Dv=64, M=4, score=0, algo=0, scale=1.0)
    assert L.kata_attn_fwd(a, None) == -1  # null pointers
    a = _lib.AttnFwdArgs(q=16, k=16, v=16, o=24, den=16, dtype=1, B=1, T=8, H=1, HQ=1, D=64, Dv=64, M=4, score=0,
                         algo=0, scale=1.0)
    assert L.kata_attn_fwd(a, None) == -4  # misaligned o
    b = _lib.AttnBwdArgs(q=16, k=16, v=16, o=16, den=16, dout=16, dq=16, dk=16, dv=16, dtype=1, B=2, T=8, H=1, HQ=2,
                         D=64, Dv=64, M=4, score=0, algo=0, scale=1.0)
    # delta (B*T*HQ) + two head-major arrays with rows padded to 128 (B*HQ*roundup(T,128)), fp32
    assert L.kata_attn_bwd_workspace_bytes(b) == 4 * (2 * 8 * 2 + 2 * 2 * 2 * 128)
    assert L.kata_attn_bwd(b, None) == -5  # workspace missing
    b.c = 16
    assert L.kata_attn_bwd(b, None) == -1  # decay without dc


def test_algo_query_reports_the_kernel_family(L):
    from linatt_b200 import _lib

    def algo(**kw):
        base = dict(dtype=1, B=1, T=8, H=1, HQ=1, D=128, Dv=128, M=4, score=0, algo=0, scale=1.0)
        base.update(kw)
        return L.kata_attn_algo(_lib.AttnFwdArgs(**base))

    assert algo() == 1                      # bf16 in the envelope: tcgen05
    assert algo(dtype=0) == 2               # fp32: the fp32-exact CUDA-core kernels
    assert algo(D=256) == 2                 # offset-gated width D != Dv: outside the envelope
    assert algo(D=256, algo=1) == -8        # forcing tensor cores there is refused
    assert algo(M=3) == -3


def test_gram_form_host_logic(L):
    """The sum score with groups of 16 (bf16, Dv = 64) runs on Gram features: algo query, workspace
    sizes (bf16 features of q and k; the backward adds their gradients after the parts-form arrays)
    and the refusals of a forced TC_GRAM outside its envelope or without its workspace."""
    from linatt_b200 import _lib

    kw = dict(dtype=1, B=2, T=8, H=1, HQ=2, D=64, Dv=64, M=4, score=1, algo=0, scale=1.0)
    al = lambda x: (x + 255) // 256 * 256  # noqa: E731
    phi = al(2 * 8 * 2 * 144 * 2) + al(2 * 8 * 1 * 144 * 2)
    a = _lib.AttnFwdArgs(**kw)
    assert L.kata_attn_algo(a) == 3
    assert L.kata_attn_fwd_workspace_bytes(a) == phi
    assert L.kata_attn_algo(_lib.AttnFwdArgs(**{**kw, "D": 128, "M": 8})) == 3  # groups of 16 at D = 128
    for other in (dict(score=0), dict(dtype=2), dict(M=2), dict(Dv=128), dict(algo=1), dict(algo=2)):
        b = _lib.AttnFwdArgs(**{**kw, **other})
        assert L.kata_attn_fwd_workspace_bytes(b) == 0, other
        assert L.kata_attn_algo(b) != 3, other
    assert L.kata_attn_algo(_lib.AttnFwdArgs(**{**kw, "score": 0, "algo": 3})) == -8
    a = _lib.AttnFwdArgs(q=16, k=16, v=16, o=16, den=16, **{**kw, "algo": 3})
    assert L.kata_attn_fwd(a, None) == -5  # TC_GRAM without its workspace
    a = _lib.AttnFwdArgs(q=16, k=16, v=16, o=16, den=16, **{**kw, "algo": 3, "score": 0})
    assert L.kata_attn_fwd(a, None) == -8  # TC_GRAM on the concat score
    base = 4 * (2 * 8 * 2 + 2 * 2 * 2 * 128)
    b = _lib.AttnBwdArgs(**kw)
    assert L.kata_attn_bwd_workspace_bytes(b) == al(base) + 2 * phi
    b.algo = 1
    assert L.kata_attn_bwd_workspace_bytes(b) == base
    b = _lib.AttnBwdArgs(q=16, k=16, v=16, o=16, den=16, dout=16, dq=16, dk=16, dv=16, **{**kw, "algo": 3})
    b.workspace, b.workspace_bytes = 256, base  # the parts-form size is not enough for TC_GRAM
    assert L.kata_attn_bwd(b, None) == -5


def test_packed_documents_host_logic(L):
    """cu_seqlens (packed documents): B = 1 and the tensor-core parts form only (with or without
    decay); the backward's workspace grows by one 128-row tile of per-query vectors per document."""
    from linatt_b200 import _lib

    kw = dict(dtype=1, B=1, T=1000, H=2, HQ=2, D=128, Dv=128, M=4, score=0, algo=0, scale=1.0,
              cu_seqlens=16, num_seqs=5)
    assert L.kata_attn_algo(_lib.AttnFwdArgs(**kw)) == 1
    assert L.kata_attn_algo(_lib.AttnFwdArgs(**{**kw, "B": 2})) == -3
    assert L.kata_attn_algo(_lib.AttnFwdArgs(**{**kw, "num_seqs": 0})) == -3
    assert L.kata_attn_algo(_lib.AttnFwdArgs(**{**kw, "dtype": 0})) == -8      # fp32
    assert L.kata_attn_algo(_lib.AttnFwdArgs(**{**kw, "algo": 2})) == -8       # SIMT
    assert L.kata_attn_algo(_lib.AttnFwdArgs(**{**kw, "c": 16})) == 1          # decay: tensor cores too
    # a sum score with groups of 16 stays on the parts form (no Gram features for packed documents)
    g = {**kw, "D": 64, "Dv": 64, "score": 1}
    assert L.kata_attn_algo(_lib.AttnFwdArgs(**g)) == 1
    assert L.kata_attn_fwd_workspace_bytes(_lib.AttnFwdArgs(**g)) == 0
    b = _lib.AttnBwdArgs(**{n: v for n, v in kw.items()})
    tiles = (1000 + 127) // 128 + 5
    assert L.kata_attn_bwd_workspace_bytes(b) == 4 * (1000 * 2 + 2 * 2 * tiles * 128)


def test_bf16_outside_the_envelope_warns_once(monkeypatch):
    import linatt_b200.parallel_kata_attn as pka
    from linatt_b200 import _lib

    monkeypatch.setattr(pka, "_SIMT_WARNED", set())
    a = _lib.AttnFwdArgs(dtype=1, B=1, T=8, H=1, HQ=1, D=256, Dv=128, M=4, score=0, algo=0, scale=1.0)
    with pytest.warns(RuntimeWarning, match="outside the tensor-core envelope"):
        pka._warn_if_simt(a, pka.torch.bfloat16)
    import warnings

    with warnings.catch_warnings():
        warnings.simplefilter("error")
        pka._warn_if_simt(a, pka.torch.bfloat16)  # second time: silent
        a.D, a.Dv = 128, 128
        pka._warn_if_simt(a, pka.torch.bfloat16)  # tensor-core shape: silent


def test_noalloc_accepts_only_the_full_backward(L):
    from linatt_b200 import _lib

    # phases 1 and 2 would split the backward across calls that share the library's one scratch
    # array, so the dk/dv pass could read another call's delta and 1/den: both are refused on the host
    for phases in (1, 2):
        b = _lib.AttnBwdArgs(q=16, k=16, v=16, o=16, den=16, dout=16, dq=16, dk=16, dv=16, dtype=1, B=1, T=8, H=1,
                             HQ=1, D=64, Dv=64, M=4, score=0, algo=0, scale=1.0, phases=phases)
        assert L.kata_attn_bwd_noalloc(b, None) == -1


def test_delta_host_side_validation(L):
    from linatt_b200 import _lib

    assert L.kata_delta_fwd(None, None) == -1
    a = _lib.DeltaFwdArgs(dtype=5, B=1, T=8, H=1, D=64, Dv=64, M=4, scale=1.0)
    assert L.kata_delta_fwd(a, None) == -2
    a = _lib.DeltaFwdArgs(dtype=1, B=1, T=8, H=1, D=64, Dv=64, M=3, scale=1.0)
    assert L.kata_delta_fwd(a, None) == -3  # D % M
    a = _lib.DeltaFwdArgs(dtype=1, B=1, T=8, H=1, D=64, Dv=64, M=8, scale=1.0)
    assert L.kata_delta_fwd(a, None) == -8  # M*M > 16
    a = _lib.DeltaFwdArgs(dtype=1, B=1, T=8, H=1, D=64, Dv=64, M=4, scale=1.0)
    assert L.kata_delta_fwd(a, None) == -1  # null pointers
    a = _lib.DeltaFwdArgs(q=16, k=16, v=16, beta=16, U=16, dtype=1, B=1, T=8, H=1, D=64, Dv=64, M=4, phases=3)
    assert L.kata_delta_fwd(a, None) == -1  # bad phases
    b = _lib.DeltaBwdArgs(q=16, k=16, v=16, beta=16, U=16, o=16, den=16, dout=16, dq=16, dk=16, dv=16, dbeta=16,
                          dtype=1, B=2, T=8, H=3, D=64, Dv=32, M=4)
    assert L.kata_delta_bwd_workspace_bytes(b) > 4 * 48 * (64 + 32)  # at least Tm and Y
    assert L.kata_delta_bwd(b, None) == -5
    f = _lib.DeltaFwdArgs(q=16, k=16, v=16, beta=16, U=16, o=16, den=16, dtype=1, B=2, T=8, H=3, D=64, Dv=32, M=4)
    assert L.kata_delta_fwd_workspace_bytes(f) > 0
    assert L.kata_delta_fwd(f, None) == -5
    b.o = None
    b.normalize = 1
    assert L.kata_delta_bwd(b, None) == -1  # normalised path needs o, den unless z is given


def test_product_path_refuses_cpu_tensors():
    import torch

    from linatt_b200.parallel_kata_attn import parallel_kata_attn

    q = torch.randn(1, 8, 1, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        parallel_kata_attn(q, q, q, num_groups=4)

    from linatt_b200.spd import flash_delta

    with pytest.raises(RuntimeError, match="CUDA"):
        flash_delta(q, q, q, q[..., 0], 4)


def test_binding_signatures_match_the_header(L):
    """Every entry point the ctypes binding types has the header's parameter kinds, in order
    (pointer / int / float): a miscounted argument list would pass garbage through the C ABI."""
    import ctypes
    import re

    from linatt_b200 import _lib

    header = (ROOT / "include" / "kata_b200.h").read_text()
    checked = 0
    for m in re.finditer(r"KATA_API\s+[\w\s\*]+?\b(kata_\w+)\s*\((.*?)\);", header, re.S):
        name, params = m.group(1), m.group(2).strip()
        fn = getattr(L, name)
        if fn.argtypes is None:
            continue
        kinds = "" if params in ("", "void") else "".join(
            "p" if ("*" in x or "kata_stream_t" in x) else ("f" if x.strip().startswith("float") else "i")
            for x in params.split(","))
        ints = (_lib.c_int, _lib.c_size_t, ctypes.c_longlong)
        bound = "".join("f" if t is _lib.c_float else ("p" if t in (_lib.c_void_p, ) or hasattr(t, "_type_")
                                                       and t not in ints else "i")
                        for t in fn.argtypes)
        assert kinds == bound, f"{name}: header {kinds} vs binding {bound}"
        checked += 1
    assert checked >= 15
