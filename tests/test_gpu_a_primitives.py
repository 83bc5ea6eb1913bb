"""Device check of the tcgen05 / TMA encodings (shared-memory descriptors for every swizzle and
major-ness, TMEM-sourced A operand) used by the attention kernels, against a plain GEMM."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

# (N, K, a_mn, b_mn, a_sw, b_sw, a_tmem)
CASES = [
    (128, 128, 0, 0, 128, 128, 0),
    (128, 64, 0, 0, 64, 64, 0),
    (128, 32, 0, 0, 32, 32, 0),
    (64, 128, 0, 0, 128, 64, 0),
    (128, 128, 0, 1, 128, 128, 0),
    (64, 128, 0, 1, 128, 128, 0),
    (32, 128, 0, 1, 128, 64, 0),
    (16, 64, 0, 1, 64, 32, 0),
    (128, 128, 1, 0, 128, 128, 0),
    (128, 64, 1, 1, 128, 128, 0),
    (256, 64, 0, 0, 128, 128, 0),
    (128, 128, 0, 0, 128, 128, 1),
    (128, 64, 0, 1, 128, 128, 1),
    (32, 128, 0, 1, 128, 64, 1),
    # Gram-feature operands (32-byte swizzle, boxes of 16 columns): the K = 144 score product and
    # the N = 144 gradient chain with its A operand in tensor memory
    (128, 144, 0, 0, 32, 32, 0),
    (144, 128, 0, 1, 128, 32, 1),
    (144, 128, 0, 1, 128, 32, 0),
]


@pytest.mark.parametrize("N,K,a_mn,b_mn,a_sw,b_sw,a_tmem", CASES)
def test_umma_selftest(N, K, a_mn, b_mn, a_sw, b_sw, a_tmem):
    from linatt_b200 import _lib

    L = _lib.lib()
    M = 128
    g = torch.Generator(device="cuda").manual_seed(N * 1000 + K)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    B = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    As = A.t().contiguous() if a_mn else A.contiguous()
    Bs = B.t().contiguous() if b_mn else B.contiguous()
    D = torch.full((M, N), float("nan"), device="cuda")
    rc = L.kata_selftest_umma(As.data_ptr(), Bs.data_ptr(), D.data_ptr(), M, N, K, a_mn, b_mn, a_sw, b_sw, a_tmem,
                              torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "kata_selftest_umma")
    torch.cuda.synchronize()
    ref = A.float() @ B.float().t()
    err = (D - ref).norm() / ref.norm()
    assert torch.isfinite(D).all()
    assert err < 1e-5, f"rel err {err.item():.3e}"


# (N, K, a_mn, b_mn, lane_off): the M = 64 tiles of the tensor-core gated delta rule
CASES64 = [(64, 64, 0, 0, 0), (64, 64, 0, 0, 16), (64, 64, 1, 0, 0), (64, 64, 0, 1, 16), (64, 64, 1, 1, 0),
           (128, 64, 0, 0, 16), (64, 128, 0, 1, 0), (64, 64, 1, 0, 16), (64, 64, 1, 1, 16), (64, 128, 1, 0, 16)]


@pytest.mark.parametrize("N,K,a_mn,b_mn,lane_off", CASES64)
def test_umma_selftest_m64(N, K, a_mn, b_mn, lane_off):
    from linatt_b200 import _lib

    L = _lib.lib()
    M = 64
    g = torch.Generator(device="cuda").manual_seed(N * 7 + K + lane_off)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    B = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    As = A.t().contiguous() if a_mn else A.contiguous()
    Bs = B.t().contiguous() if b_mn else B.contiguous()
    D = torch.full((M, N), float("nan"), device="cuda")
    rc = L.kata_selftest_umma_m64(As.data_ptr(), Bs.data_ptr(), D.data_ptr(), N, K, a_mn, b_mn, lane_off,
                                  torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "kata_selftest_umma_m64")
    torch.cuda.synchronize()
    ref = A.float() @ B.float().t()
    assert torch.isfinite(D).all()
    err = (D - ref).norm() / ref.norm()
    assert err < 1e-5, f"rel err {err.item():.3e}"


# (N, K, a_mn, b_mn, a_sw, b_sw, a_tmem): CTA-pair (cta_group::2, M = 256) tiles of the attention
# kernels -- B halves split by N across the two CTAs.
CASES_PAIR = [
    (128, 128, 0, 0, 128, 128, 0),   # score part: K-major A and B
    (128, 32, 0, 0, 64, 64, 0),      # one E = 32 group (64-byte swizzle)
    (128, 128, 0, 1, 128, 128, 0),   # MN-major B (a V or dO tile), 64 columns per CTA
    (64, 128, 0, 1, 128, 64, 0),     # MN-major B, 32 columns per CTA
    (32, 128, 0, 1, 128, 32, 0),     # N = 32 (a gradient chain of one group), 16 columns per CTA
    (128, 128, 0, 1, 128, 128, 1),   # A from tensor memory (P or W operand)
    (32, 128, 0, 1, 128, 32, 1),
    (256, 64, 0, 0, 128, 128, 0),
    (128, 128, 1, 0, 128, 128, 0),   # MN-major A
]


@pytest.mark.parametrize("N,K,a_mn,b_mn,a_sw,b_sw,a_tmem", CASES_PAIR)
def test_umma_selftest_pair(N, K, a_mn, b_mn, a_sw, b_sw, a_tmem):
    from linatt_b200 import _lib

    L = _lib.lib()
    M = 256
    g = torch.Generator(device="cuda").manual_seed(N * 31 + K + 7 * a_tmem)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    B = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    As = A.t().contiguous() if a_mn else A.contiguous()
    Bs = B.t().contiguous() if b_mn else B.contiguous()
    D = torch.full((M, N), float("nan"), device="cuda")
    rc = L.kata_selftest_umma_pair(As.data_ptr(), Bs.data_ptr(), D.data_ptr(), N, K, a_mn, b_mn, a_sw, b_sw, a_tmem,
                                   torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "kata_selftest_umma_pair")
    torch.cuda.synchronize()
    ref = A.float() @ B.float().t()
    assert torch.isfinite(D).all()
    err = (D - ref).norm() / ref.norm()
    assert err < 1e-5, f"rel err {err.item():.3e}"
