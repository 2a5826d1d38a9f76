"""GPU parity of the many-token (persistent, tokens-as-M) tcgen05 GEMM path.

Projections with more than 128 tokens (prefix LM, SigLIP, batched denoise) run on
the wide kernel; these cases cover its tile widths (128 / 256), ragged token and
column edges, the split-K ticket reduction and every fused epilogue, against fp32
torch references on the same bf16 inputs (tolerance: bf16 output rounding plus
fp32 summation-order noise).
"""

import pytest
import torch

from pi05_infer import ops

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _bf(x):
    return x.to(torch.bfloat16)


def _close(got, ref, rtol=1.6e-2, atol=2e-3):
    got = got.float()
    err = (got - ref).abs()
    lim = atol + rtol * ref.abs()
    bad = (err > lim).sum().item()
    assert bad == 0, f"{bad} mismatches, max err {err.max().item():.3e}, max ref {ref.abs().max().item():.3e}"


def gelu_tanh(x):
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)))


@pytest.mark.parametrize("m,n,k", [(129, 4096, 1024), (300, 4160, 1024), (968, 16384, 2048)])
def test_wide_geglu(m, n, k):
    g = torch.Generator(device=DEV).manual_seed(10)
    x = _bf(torch.randn(m, k, device=DEV, generator=g))
    wg = _bf(torch.randn(n, k, device=DEV, generator=g) * 0.02)
    wu = _bf(torch.randn(n, k, device=DEV, generator=g) * 0.02)
    out = ops.geglu(x, wg, wu)
    gg = (x.float() @ wg.float().t()).bfloat16().float()
    uu = x.float() @ wu.float().t()
    _close(out, gelu_tanh(gg) * uu)
    assert ops.read_device_status() == 0


@pytest.mark.parametrize("m,n,k", [(200, 2560, 1024), (768, 3456, 1152), (768, 1152, 4352), (968, 2048, 16384),
                                   (1000, 1152, 1152)])
def test_wide_linear(m, n, k):
    g = torch.Generator(device=DEV).manual_seed(11)
    x = _bf(torch.randn(m, k, device=DEV, generator=g))
    w = _bf(torch.randn(n, k, device=DEV, generator=g) * 0.02)
    out = ops.linear(x, w)
    _close(out, x.float() @ w.float().t(), atol=4e-3)
    assert ops.read_device_status() == 0
    # deterministic: a second launch (split-K tickets re-armed) gives identical bits
    out2 = ops.linear(x, w)
    assert torch.equal(out, out2)


@pytest.mark.parametrize("m,n,k", [(968, 2048, 2048), (968, 2048, 16384), (768, 1152, 4352)])
def test_wide_gated_residual(m, n, k):
    g = torch.Generator(device=DEV).manual_seed(12)
    x = _bf(torch.randn(m, k, device=DEV, generator=g))
    w = _bf(torch.randn(n, k, device=DEV, generator=g) * 0.02)
    resid = _bf(torch.randn(m, n, device=DEV, generator=g))
    gate = torch.randn(n, device=DEV, generator=g)
    out = ops.linear_gated_residual(x, w, resid, gate)
    y = (x.float() @ w.float().t()).bfloat16().float()
    _close(out, resid.float() + y * gate.bfloat16().float(), atol=2e-2)
    r2 = resid.clone()
    ops.linear_gated_residual(x, w, r2, None, out=r2)  # in place, no gate
    _close(r2, resid.float() + y, atol=2e-2)
    assert ops.read_device_status() == 0


def _rope_ref(x, cos, sin):
    half = x.shape[-1] // 2
    lo, hi = x[..., :half], x[..., half:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([lo * c[..., :half] - hi * s[..., :half], hi * c[..., half:] + lo * s[..., half:]], -1)


def _rope_mag(x, cos, sin):
    """|lo||c| + |hi||s| per output: the scale of one bf16 ulp flip of the rounded
    projection (the kernel and the reference may round a near-tie differently)."""
    half = x.shape[-1] // 2
    lo, hi = x[..., :half].abs(), x[..., half:].abs()
    c, s = cos[:, None, :].abs(), sin[:, None, :].abs()
    return torch.cat([lo * c[..., :half] + hi * s[..., :half], hi * c[..., half:] + lo * s[..., half:]], -1)


def _close_rope(got, ref, mag):
    err = (got.float() - ref).abs()
    lim = 2e-3 + 1.6e-2 * mag
    bad = (err > lim).sum().item()
    assert bad == 0, f"{bad} mismatches, max err {err.max().item():.3e}"


@pytest.mark.parametrize("m,krow0,k", [(968, 0, 2048), (300, 50, 1024)])
def test_wide_qkv_rope(m, krow0, k):
    g = torch.Generator(device=DEV).manual_seed(13)
    hq, hkv, d = 8, 1, 256
    x = _bf(torch.randn(m, k, device=DEV, generator=g))
    w = _bf(torch.randn((hq + 2 * hkv) * d, k, device=DEV, generator=g) * 0.02)
    pos = torch.arange(krow0, krow0 + m, device=DEV).float()
    inv = 1.0 / (10000 ** (torch.arange(0, d, 2, device=DEV).float() / d))
    fr = pos[:, None] * inv[None]
    emb = torch.cat([fr, fr], -1)
    cos, sin = _bf(emb.cos()), _bf(emb.sin())
    kv_rows = krow0 + m + 16
    kc = torch.zeros(1, kv_rows, d, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros(1, kv_rows, d, dtype=torch.bfloat16, device=DEV)
    q = torch.empty(m, hq, d, dtype=torch.bfloat16, device=DEV)
    ops.qkv_rope(x, w, cos, sin, q, kc, vc, krow0, hq, hkv, d)
    qkv = (x.float() @ w.float().t()).bfloat16().float()
    qr = _rope_ref(qkv[:, : hq * d].view(m, hq, d), cos.float(), sin.float())
    kr = _rope_ref(qkv[:, hq * d: (hq + 1) * d].view(m, 1, d), cos.float(), sin.float())[:, 0]
    vr = qkv[:, (hq + 1) * d:]
    qm = _rope_mag(qkv[:, : hq * d].view(m, hq, d), cos.float(), sin.float())
    km = _rope_mag(qkv[:, hq * d: (hq + 1) * d].view(m, 1, d), cos.float(), sin.float())[:, 0]
    _close_rope(q, qr, qm)
    _close_rope(kc[0, krow0: krow0 + m], kr, km)
    _close(vc[0, krow0: krow0 + m], vr)
    assert kc[0, :krow0].abs().sum().item() == 0  # rows outside [krow0, krow0 + m) untouched
    assert kc[0, krow0 + m:].abs().sum().item() == 0
    assert ops.read_device_status() == 0
