"""GPU parity of the sequence-parallel KATA-SPD path.  On one GPU the ranks are emulated (each
shard's pieces run in turn, prefix / suffix sums formed by hand) and the result is compared with the
single-GPU kernels over the whole sequence and with the fp64 oracle; with two or more GPUs the real
NCCL path runs under torchrun (tests/sp_worker.py).  Tolerance (relative L2): 1e-2, bf16 inputs."""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from oracle import kata_oracle as ko

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def draw(seed, B, T, H, D, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(B, T, H, D, generator=g) / D ** 0.5 for _ in range(3))
    do = torch.randn(B, T, H, D, generator=g)
    return tuple(x.to(dtype).cuda() for x in (q, k, v, do))


def emulate(q, k, v, do, R, M):
    """Sequence-parallel forward + backward over R emulated ranks on one GPU."""
    from linatt_b200 import sequence_parallel as sp

    return sp.sp_emulate(q, k, v, do, R, M)


def full(q, k, v, do, M):
    import linatt_b200.parallel_kata_attn as pka

    q, k, v = (x.detach().clone().requires_grad_(True) for x in (q, k, v))
    o, den = pka._fwd(q, k, v, M, None, "concat")
    dq, dk, dv, _ = pka._bwd(q, k, v, o, den, do, M, None, "concat")
    return o, den, dq, dk, dv


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm())


@pytest.mark.parametrize("R,M,T", [(2, 4, 1024), (3, 4, 1536), (4, 2, 2048)])
def test_sp_emulated_matches_single_gpu(R, M, T):
    q, k, v, do = draw(R * 10 + M, 1, T, 2, 128)
    o, D, dq, dk, dv = emulate(q, k, v, do, R, M)
    fo, fden, fdq, fdk, fdv = full(q, k, v, do, M)
    assert rel(D, fden) < 1e-2
    for name, a, b in (("o", o, fo), ("dq", dq, fdq), ("dk", dk, fdk), ("dv", dv, fdv)):
        e = rel(a, b)
        assert e < 1e-2, f"{name}: rel-L2 {e:.3e}"


def test_sp_emulated_matches_oracle():
    B, T, H, D, M, R = 1, 768, 2, 128, 4, 3
    q, k, v, do = draw(77, B, T, H, D)
    o, _, dq, dk, dv = emulate(q, k, v, do, R, M)
    f = lambda x: x.float().cpu().double().numpy()
    ro, _ = ko.attn_fwd(f(q), f(k), f(v), M, (D // M) ** -0.5)
    rdq, rdk, rdv, _ = ko.attn_bwd(f(q), f(k), f(v), f(do), M, (D // M) ** -0.5)
    assert ko.rel_l2(f(o), ro) < 1e-2
    for name, g, r in (("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
        assert ko.rel_l2(f(g), r) < 1e-2, name


def test_config4_full_size_emulated_ranks():
    """Config 4 at its size (B=1, T=131072, H=16, D=Dv=128, M=4, bf16): R in {2, 4, 8} emulated
    ranks against the single-GPU kernels over the whole sequence (o, den, dq, dk, dv), and both
    against the exact fp64 oracle on the last 256 tokens of two heads.  At this length the
    cross-shard state sums up to 114 688 tokens in fp32 before the bf16 GEMM; the tail window is
    where that matters most (its queries see every earlier shard)."""
    B, T, H, D, M = 1, 131072, 16, 128, 4
    g = torch.Generator(device="cuda").manual_seed(44)
    q, k, v = ((torch.randn(B, T, H, D, device="cuda", generator=g) / D ** 0.5).bfloat16() for _ in range(3))
    do = torch.randn(B, T, H, D, device="cuda", generator=g).bfloat16()
    ref = full(q, k, v, do, M)
    torch.cuda.synchronize()
    w = 256
    f = lambda x, h: x[0, :, h].float().cpu().numpy()  # noqa: E731
    oracle = {h: ko.attn_tail_window(f(q, h), f(k, h), f(v, h), f(do, h), M, w) for h in (0, 15)}

    def check_tail(outs, tag):
        for h, r in oracle.items():
            for name, got in zip(("o", "den", "dq", "dk", "dv"), outs):
                x = got[0, T - w:, h].float().cpu().numpy()
                e = ko.rel_l2(x, r[name])
                assert e < 1e-2, f"{tag} head {h} tail {name}: rel-L2 {e:.3e}"

    check_tail(ref, "single GPU")
    for R in (2, 4, 8):
        got = emulate(q, k, v, do, R, M)
        for name, a, b in zip(("o", "den", "dq", "dk", "dv"), got, ref):
            e = rel(a, b)
            assert e < 1e-2, f"R={R} {name}: rel-L2 {e:.3e} against the single-GPU kernels"
        check_tail(got, f"R={R}")
        del got
        torch.cuda.empty_cache()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs (the real NCCL path)")
def test_sp_nccl_two_ranks():
    n = min(torch.cuda.device_count(), 4)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", "--master-port", "29531", str(ROOT / "tests" / "sp_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "SP_OK" in r.stdout


@pytest.mark.parametrize("D,M,dtype,accumulate", [(128, 4, torch.bfloat16, 0), (64, 4, torch.float32, 1),
                                                  (128, 2, torch.float16, 1), (96, 4, torch.bfloat16, 0),
                                                  (256, 8, torch.bfloat16, 1)])
def test_feature_gradient_contraction_vs_torch(D, M, dtype, accumulate):
    """kata_sp_contract: dx_{g,a} (+)= factor * sum_b G[g,b,a] x_{g,b} against torch fp32 (rel-L2
    <= 1e-5), on the 16-byte path (E = 16, 32, 64) and the general one (E = 24)."""
    from linatt_b200 import _lib

    B, T, H = 2, 37, 3
    E = D // M
    g = torch.Generator().manual_seed(D * M + accumulate)
    x = torch.randn(B, T, H, D, generator=g).to(dtype).cuda()
    G = torch.randn(B * H, T, M * E * E, generator=g).bfloat16().cuda()
    dx0 = torch.randn(B, T, H, D, generator=g).cuda()
    dx = dx0.clone()
    factor = 0.37
    _lib.check(_lib.lib().kata_sp_contract(G.data_ptr(), x.data_ptr(), dx.data_ptr(), _lib.DTYPE[dtype], B, T, H, D,
                                           M, factor, accumulate, torch.cuda.current_stream().cuda_stream),
               "kata_sp_contract")
    Gr = G.float().view(B, H, T, M, E, E)  # [.., g, b, a]
    xr = x.float().permute(0, 2, 1, 3).reshape(B, H, T, M, E)
    ref = factor * torch.einsum("bhtgca,bhtgc->bhtga", Gr, xr).reshape(B, H, T, D).permute(0, 2, 1, 3)
    if accumulate:
        ref = ref + dx0
    assert ko.rel_l2(dx.cpu().numpy(), ref.cpu().numpy()) < 1e-5
