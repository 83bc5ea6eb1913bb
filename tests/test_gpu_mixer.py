"""Mixer prologue / epilogue kernels (short convolution, row normalisation with RoPE) and the whole
FlashKata mixer on the GPU.

* kernels against float64 PyTorch statements of the same operations (fp32 at rel-L2 <= 1e-5,
  16-bit at <= 1e-2), including strided inputs, ragged T and every RoPE form;
* the mixer against the golden fixtures made by running the reference's own ``KataAttention``
  forward / backward (``tests/golden/make_golden_mixer.py``): output, input gradient and every
  parameter gradient, fp32 at rel-L2 <= 1e-5;
* the config-5 mixer geometry in bf16 against the same mixer in fp32 (<= 1e-2), and one
  optimisation step of a small KATA LM.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).parent / "golden" / "mixer_golden.npz"


def rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def conv_ref(x, w, act):
    T = x.shape[1]
    y = F.conv1d(x.transpose(1, 2), w, padding=w.shape[-1] - 1, groups=x.shape[-1])[..., :T].transpose(1, 2)
    return F.silu(y) if act else y


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("K", [1, 2, 3, 4])
@pytest.mark.parametrize("T", [1, 63, 64, 65, 200])
@pytest.mark.parametrize("act", [True, False])
def test_short_conv(dtype, K, T, act):
    from linatt_b200.mixer import ShortConvQKVFunction

    g = torch.Generator(device="cuda").manual_seed(K * 1000 + T)
    B, C1, C2 = 2, 48, 32
    xf = torch.randn(B, T, C1 + C2, device="cuda", generator=g)
    w1 = torch.randn(C1, 1, K, device="cuda", generator=g) * 0.5
    w2 = torch.randn(C2, 1, K, device="cuda", generator=g) * 0.5
    x = xf.to(dtype).requires_grad_(True)
    w1.requires_grad_(True), w2.requires_grad_(True)
    y1, y2 = ShortConvQKVFunction.apply(x, act, w1, w2)
    dy1 = torch.randn_like(y1.float()).to(dtype)
    dy2 = torch.randn_like(y2.float()).to(dtype)
    torch.autograd.backward([y1, y2], [dy1, dy2])
    xd = x.detach().double().requires_grad_(True)
    w1d, w2d = (w.detach().double().requires_grad_(True) for w in (w1, w2))
    r1, r2 = conv_ref(xd[..., :C1], w1d, act), conv_ref(xd[..., C1:], w2d, act)
    torch.autograd.backward([r1, r2], [dy1.double(), dy2.double()])
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    for a, b in ((y1, r1), (y2, r2), (x.grad, xd.grad), (w1.grad, w1d.grad), (w2.grad, w2d.grad)):
        assert torch.isfinite(a).all()
        assert rel(a, b) < tol


def rot_ref(x, cos, sin, rope, R):
    # fla rotary_embedding_ref semantics: interleaved pairs over the row (rope 1) or the
    # half rotation inside groups of R values (rope 2)
    B, T, H, D = x.shape
    c, s = cos[:T].double(), sin[:T].double()
    if rope == 1:
        c2 = c.repeat_interleave(2, -1)[None, :, None, :]
        s2 = s.repeat_interleave(2, -1)[None, :, None, :]
        x1, x2 = x[..., ::2], x[..., 1::2]
        rh = torch.stack((-x2, x1), dim=-1).reshape(x.shape)
        return x * c2 + rh * s2
    xg = x.reshape(B, T, H, D // R, R)
    c2 = torch.cat([c, c], -1)[None, :, None, None, :]
    s2 = torch.cat([s, s], -1)[None, :, None, None, :]
    x1, x2 = xg[..., : R // 2], xg[..., R // 2:]
    rh = torch.cat((-x2, x1), -1)
    return (xg * c2 + rh * s2).reshape(B, T, H, D)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("norm", ["none", "l2", "rms", "rms_noweight"])
@pytest.mark.parametrize("rope,R", [(0, 0), (1, 64), (2, 16), (2, 32)])
def test_row_norm_rope(dtype, norm, rope, R):
    from linatt_b200.mixer import RowNormFunction, rope_tables

    if norm == "none" and rope == 0:
        pytest.skip("identity")
    B, T, H, D = 2, 70, 3, 64
    g = torch.Generator(device="cuda").manual_seed(hash((norm, rope, R)) % 1000)
    x = torch.randn(B, T, H, D, device="cuda", generator=g).to(dtype).requires_grad_(True)
    w = (1 + 0.3 * torch.randn(D, device="cuda", generator=g)).requires_grad_(True)
    code = {"none": 0, "l2": 1, "rms": 2, "rms_noweight": 2}[norm]
    wt = w if norm == "rms" else None
    eps = 1e-6 if norm == "l2" else 1e-5
    cos = sin = None
    if rope:
        cos, sin = rope_tables(T, R, 10000.0, "cuda", dtype)
    y = RowNormFunction.apply(x.reshape(-1, D), wt, cos, sin, code, rope, R or D, eps, H, T).view(B, T, H, D)
    dy = torch.randn(B, T, H, D, device="cuda", generator=g).to(dtype)
    y.backward(dy)
    xd = x.detach().double().requires_grad_(True)
    wd = w.detach().double().requires_grad_(True)
    r = xd
    if code == 1:
        r = r * torch.rsqrt(r.pow(2).sum(-1, keepdim=True) + eps)
    elif code == 2:
        r = r * torch.rsqrt(r.pow(2).mean(-1, keepdim=True) + eps)
        if norm == "rms":
            r = r * wd
    if rope:
        r = rot_ref(r, cos, sin, rope, R)
    r.backward(dy.double())
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert rel(y, r) < tol
    assert rel(x.grad, xd.grad) < tol
    if norm == "rms":
        assert rel(w.grad, wd.grad) < tol


def _golden_cases():
    if not GOLDEN.exists():
        return []
    z = np.load(GOLDEN)
    return sorted({k.split("/")[0] for k in z.files})


GOLDEN_KW = {
    "conv_m4": dict(hidden_size=128, num_heads=2, spd_num_groups=4, use_short_conv=True, norm_eps=1e-6),
    "l2_rope_m2": dict(hidden_size=128, num_heads=2, spd_num_groups=2, use_short_conv=True, qk_norm=True,
                       norm_q="l2", norm_k="l2", use_rope=True),
    "rms_ropegroup_m4": dict(hidden_size=128, num_heads=2, spd_num_groups=4, qk_norm=True, norm_q="rmsnorm",
                             norm_k="rmsnorm", use_rope=True, rope_group=True),
    "decay_conv_m2": dict(hidden_size=128, num_heads=2, spd_num_groups=2, use_short_conv=True, use_decay=True),
    "offset_m4": dict(hidden_size=128, num_heads=2, spd_num_groups=4, use_offset_gate=True),
    "gqa_conv_m4": dict(hidden_size=128, num_heads=4, num_kv_heads=2, spd_num_groups=4, use_short_conv=True,
                        expand_k=2.0, expand_v=2.0),
}


@pytest.mark.parametrize("case", _golden_cases())
def test_mixer_golden_fp32(case):
    """fp32 mixer against the reference layer's own forward / backward (float64 on CPU)."""
    from linatt_b200.mixer import FlashKataMixer

    z = np.load(GOLDEN)
    get = lambda k: torch.from_numpy(z[f"{case}/{k}"]).cuda()  # noqa: E731
    m = FlashKataMixer(feature_map="kata_quadratic", **GOLDEN_KW[case]).cuda()
    names = [k.split("/", 2)[2] for k in z.files if k.startswith(f"{case}/p/")]
    assert sorted(names) == sorted(n for n, _ in m.named_parameters())
    m.load_state_dict({n: get(f"p/{n}") for n in names}, strict=True)
    x = get("x").requires_grad_(True)
    o, _, _ = m(x)
    o.backward(get("do"))
    tol = 1e-5
    assert rel(o, get("o")) < tol, rel(o, get("o"))
    assert rel(x.grad, get("dx")) < tol, rel(x.grad, get("dx"))
    for n, p in m.named_parameters():
        e = rel(p.grad, get(f"g/{n}"))
        assert e < tol, (n, e)


def test_mixer_config5_bf16():
    """The config-5 layer (d_model 768, 12 x 64 heads, M = 4, short convolution) under bf16 autocast,
    on the tensor-core kernels, against the same parameters in fp32."""
    from linatt_b200.mixer import FlashKataMixer

    torch.manual_seed(0)
    m = FlashKataMixer(feature_map="kata_quadratic", hidden_size=768, num_heads=12, spd_num_groups=4,
                       use_short_conv=True, norm_eps=1e-6).cuda()
    x = torch.randn(2, 300, 768, device="cuda")
    do = torch.randn(2, 300, 768, device="cuda")
    xr = x.clone().requires_grad_(True)
    o32, _, _ = m(xr)
    o32.backward(do)
    g32 = {n: p.grad.clone() for n, p in m.named_parameters()}
    dx32 = xr.grad.clone()
    m.zero_grad()
    xb = x.clone().requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        ob, _, _ = m(xb)
    ob.float().backward(do)
    assert rel(ob.float(), o32) < 1e-2
    assert rel(xb.grad, dx32) < 2e-2
    for n, p in m.named_parameters():
        assert rel(p.grad, g32[n]) < 3e-2, n


def test_lm_step():
    """One AdamW step of a 2-layer KATA LM under bf16 autocast: finite loss and gradients, and the
    loss goes down over a few steps on a fixed batch."""
    from linatt_b200.lm import KataLM, KataLMConfig

    torch.manual_seed(0)
    cfg = KataLMConfig(hidden_size=256, num_hidden_layers=2, num_heads=4, vocab_size=512)
    model = KataLM(cfg).cuda()
    opt = torch.optim.AdamW(model.parameters(), lr=3e-3)
    ids = torch.randint(0, 512, (2, 256), device="cuda")
    losses = []
    for _ in range(6):
        opt.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = model(ids, labels=ids)
        loss.backward()
        assert all(torch.isfinite(p.grad).all() for p in model.parameters() if p.grad is not None)
        opt.step()
        losses.append(loss.item())
    assert all(np.isfinite(losses))
    assert losses[-1] < losses[0]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("N", [256, 512, 768, 1024])
@pytest.mark.parametrize("norm", ["l2", "rms"])
def test_row_norm_wide(dtype, N, norm):
    """Rows wider than 32 vectors (the LM's 768-wide hidden RMSNorm): one warp per row, at most six
    16-byte vectors per lane (fp32 rows up to 768 values, 16-bit rows up to 1536)."""
    from linatt_b200.mixer import RowNormFunction

    if N // (16 // torch.tensor([], dtype=dtype).element_size()) > 192:
        pytest.skip("wider than the kernel's 6 x 32 vectors")

    g = torch.Generator(device="cuda").manual_seed(N)
    rows = 1000
    x = (3 * torch.randn(rows, N, device="cuda", generator=g)).to(dtype).requires_grad_(True)
    w = (1 + 0.3 * torch.randn(N, device="cuda", generator=g)).requires_grad_(True)
    code, eps = (1, 1e-6) if norm == "l2" else (2, 1e-6)
    wt = w if norm == "rms" else None
    y = RowNormFunction.apply(x, wt, None, None, code, 0, N, eps, 1, 1)
    dy = torch.randn(rows, N, device="cuda", generator=g).to(dtype)
    y.backward(dy)
    xd = x.detach().double().requires_grad_(True)
    wd = w.detach().double().requires_grad_(True)
    if code == 1:
        r = xd * torch.rsqrt(xd.pow(2).sum(-1, keepdim=True) + eps)
    else:
        r = xd * torch.rsqrt(xd.pow(2).mean(-1, keepdim=True) + eps) * wd
    r.backward(dy.double())
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert rel(y, r) < tol
    assert rel(x.grad, xd.grad) < tol
    if norm == "rms":
        assert rel(w.grad, wd.grad) < tol


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("N", [256, 768, 1024])
def test_add_rmsnorm(dtype, N):
    """Residual add + RMSNorm against PyTorch in float64: h_out, y and the gradients of h, x and w,
    with gradients arriving both through y and through h_out's other uses."""
    from linatt_b200.lm import AddRMSNormFunction

    g = torch.Generator(device="cuda").manual_seed(N)
    rows, eps = 700, 1e-6
    h = (2 * torch.randn(rows, N, device="cuda", generator=g)).requires_grad_(True)
    x = torch.randn(rows, N, device="cuda", generator=g).to(dtype).requires_grad_(True)
    w = (1 + 0.3 * torch.randn(N, device="cuda", generator=g)).requires_grad_(True)
    h_out, y = AddRMSNormFunction.apply(h, x, w, eps)
    assert h_out.dtype == torch.float32 and y.dtype == dtype
    dh_out = torch.randn(rows, N, device="cuda", generator=g)
    dy = torch.randn(rows, N, device="cuda", generator=g).to(dtype)
    torch.autograd.backward((h_out, y), (dh_out, dy))
    hd, xd, wd = (t.detach().double().requires_grad_(True) for t in (h, x, w))
    s = hd + xd
    r = s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + eps) * wd
    torch.autograd.backward((s, r), (dh_out.double(), dy.double()))
    assert rel(h_out, s) < 1e-6
    assert rel(y, r) < 1e-2
    for got, ref, n in ((h.grad, hd.grad, "dh"), (x.grad, xd.grad, "dx"), (w.grad, wd.grad, "dw")):
        e = rel(got, ref)
        assert e < (1e-5 if n != "dx" else 1e-2), f"{n}: {e:.3e}"


def test_lm_fused_add_norm_matches_the_block_form():
    """KataLM.forward (residual adds fused with the following RMSNorm) equals the plain block-by-block
    form (KataBlock.forward, then the final norm) on the same weights: loss and gradients."""
    from linatt_b200.lm import CrossEntropyFunction, KataLM, KataLMConfig

    torch.manual_seed(1)
    cfg = KataLMConfig(hidden_size=256, num_hidden_layers=2, num_heads=4, vocab_size=512)
    model = KataLM(cfg).cuda()
    ids = torch.randint(0, 512, (2, 256), device="cuda")

    def plain(m, input_ids, labels):
        h = m.model.embeddings(input_ids)
        for blk in m.model.layers:
            h = blk(h)
        logits = m.lm_head(m.model.norm(h))
        tgt = torch.cat([labels[:, 1:], torch.full_like(labels[:, :1], -100)], dim=1)
        return CrossEntropyFunction.apply(logits.reshape(-1, logits.shape[-1]), tgt.reshape(-1))

    losses, grads = [], []
    for fn in (lambda: model(ids, labels=ids), lambda: plain(model, ids, ids)):
        model.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = fn()
        loss.backward()
        losses.append(loss.item())
        grads.append({n: p.grad.detach().clone() for n, p in model.named_parameters() if p.grad is not None})
    assert abs(losses[0] - losses[1]) < 1e-4 * abs(losses[1])
    assert grads[0].keys() == grads[1].keys()
    for n in grads[0]:
        assert rel(grads[0][n], grads[1][n]) < 2e-2, n


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_swiglu_and_cross_entropy(dtype):
    """The LM's fused SwiGLU and cross entropy against PyTorch in float64 (values and gradients),
    with ignored (-100) targets and a non-unit upstream gradient."""
    from linatt_b200.lm import CrossEntropyFunction, SwiGLUFunction

    g = torch.Generator(device="cuda").manual_seed(3)
    gu = (2 * torch.randn(300, 2 * 256, device="cuda", generator=g)).to(dtype).requires_grad_(True)
    y = SwiGLUFunction.apply(gu)
    dy = torch.randn(300, 256, device="cuda", generator=g).to(dtype)
    y.backward(dy)
    gd = gu.detach().double().requires_grad_(True)
    a, b = gd.chunk(2, -1)
    r = F.silu(a) * b
    r.backward(dy.double())
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert rel(y, r) < tol and rel(gu.grad, gd.grad) < tol
    logits = (3 * torch.randn(257, 32000, device="cuda", generator=g)).to(dtype).requires_grad_(True)
    tgt = torch.randint(0, 32000, (257,), device="cuda", generator=g)
    tgt[::7] = -100
    loss = CrossEntropyFunction.apply(logits, tgt)
    (0.5 * loss).backward()
    ld = logits.detach().double().requires_grad_(True)
    ref = F.cross_entropy(ld, tgt, ignore_index=-100)
    (0.5 * ref).backward()
    assert abs(loss.item() - ref.item()) / abs(ref.item()) < (1e-6 if dtype == torch.float32 else 1e-3)
    assert rel(logits.grad, ld.grad) < tol
