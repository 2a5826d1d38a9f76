"""GPU parity of the swap-AB tcgen05 GEMM ops against fp32 torch references.

Inputs are bf16; the reference math runs in fp32 on the same bf16 values and
rounds where the reference op rounds.  Tolerance: bf16 output rounding
(relative 1/128) plus fp32 summation-order noise.
"""

import pytest
import torch

from pi05_infer import _lib, ops

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


@pytest.fixture(params=[1, 0], ids=["splits1", "auto"])
def splits(request):
    _lib.lib().pi05_debug_set_splits(request.param)
    yield request.param
    _lib.lib().pi05_debug_set_splits(0)


def gelu_tanh(x):
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)))


@pytest.mark.parametrize("m", [50, 1, 64, 200])
def test_geglu(splits, m):
    g = torch.Generator(device=DEV).manual_seed(0)
    x = _bf(torch.randn(m, 1024, device=DEV, generator=g))
    wg = _bf(torch.randn(4096, 1024, device=DEV, generator=g) * 0.02)
    wu = _bf(torch.randn(4096, 1024, device=DEV, generator=g) * 0.02)
    out = ops.geglu(x, wg, wu)
    gg = (x.float() @ wg.float().t()).bfloat16().float()
    uu = x.float() @ wu.float().t()
    _close(out, gelu_tanh(gg) * uu)
    assert ops.read_device_status() == 0


@pytest.mark.parametrize("n,k", [(1024, 2048), (1024, 4096), (2048, 1024)])
def test_linear_gated_residual(splits, n, k):
    g = torch.Generator(device=DEV).manual_seed(1)
    m = 50
    x = _bf(torch.randn(m, k, device=DEV, generator=g))
    w = _bf(torch.randn(n, k, device=DEV, generator=g) * 0.02)
    resid = _bf(torch.randn(m, n, device=DEV, generator=g))
    gate = torch.randn(n, device=DEV, generator=g)
    out = ops.linear_gated_residual(x, w, resid, gate)
    y = (x.float() @ w.float().t()).bfloat16().float()
    ref = resid.float() + y * gate.bfloat16().float()
    # bf16 output of a sum whose operands are O(1): one bf16 ulp of the operands
    _close(out, ref, atol=2e-2)
    # in place (out aliases resid), no gate
    r2 = resid.clone()
    ops.linear_gated_residual(x, w, r2, None, out=r2)
    _close(r2, resid.float() + y, atol=2e-2)


def test_linear_plain(splits):
    g = torch.Generator(device=DEV).manual_seed(2)
    x = _bf(torch.randn(50, 1024, device=DEV, generator=g))
    w = _bf(torch.randn(2560, 1024, device=DEV, generator=g) * 0.02)
    _close(ops.linear(x, w), x.float() @ w.float().t())


def _rope_ref(x, cos, sin):
    half = x.shape[-1] // 2
    lo, hi = x[..., :half], x[..., half:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([lo * c[..., :half] - hi * s[..., :half], hi * c[..., half:] + lo * s[..., half:]], -1)


@pytest.mark.parametrize("m,krow0", [(50, 968), (50, 1430), (7, 3)])
def test_qkv_rope_kv(splits, m, krow0):
    g = torch.Generator(device=DEV).manual_seed(3)
    hq, hkv, d, k = 8, 1, 256, 1024
    x = _bf(torch.randn(m, k, device=DEV, generator=g))
    w = _bf(torch.randn((hq + 2 * hkv) * d, k, device=DEV, generator=g) * 0.02)
    pos = torch.arange(krow0, krow0 + m, device=DEV).float()
    inv = 1.0 / (10000 ** (torch.arange(0, d, 2, device=DEV).float() / d))
    fr = pos[:, None] * inv[None]
    emb = torch.cat([fr, fr], -1)
    cos, sin = _bf(emb.cos()), _bf(emb.sin())
    kv_rows = krow0 + m
    kc = torch.zeros(1, kv_rows, d, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros(1, kv_rows, d, dtype=torch.bfloat16, device=DEV)
    q = torch.empty(m, hq, d, dtype=torch.bfloat16, device=DEV)
    ops.qkv_rope(x, w, cos, sin, q, kc, vc, krow0, hq, hkv, d)
    qkv = (x.float() @ w.float().t()).bfloat16().float()
    qr = _rope_ref(qkv[:, : hq * d].view(m, hq, d), cos.float(), sin.float())
    kr = _rope_ref(qkv[:, hq * d : (hq + 1) * d].view(m, 1, d), cos.float(), sin.float())[:, 0]
    vr = qkv[:, (hq + 1) * d :]
    _close(q, qr)
    _close(kc[0, krow0:], kr)
    _close(vc[0, krow0:], vr)
    assert kc[0, :krow0].abs().sum().item() == 0  # rows before krow0 untouched


def test_reference_custom_ops_names():
    g = torch.Generator(device=DEV).manual_seed(4)
    x = _bf(torch.randn(1, 50, 1024, device=DEV, generator=g))
    wg = _bf(torch.randn(4096, 1024, device=DEV, generator=g) * 0.02)
    wu = _bf(torch.randn(4096, 1024, device=DEV, generator=g) * 0.02)
    out = torch.ops.pi05_infer.gate_up_geglu(x, wg, wu)
    assert out.shape == (1, 50, 4096)
    assert ops.fused_gate_up_geglu(x.cpu(), wg.cpu(), wu.cpu()) is None  # CPU tensors: not applicable


@pytest.mark.parametrize("m,n,k", [(768, 1152, 1152), (768, 1152, 4352), (768, 3456, 1152), (968, 2048, 2048),
                                   (600, 2048, 2048), (968, 2048, 16384)],
                         ids=["siglip_o", "siglip_fc2", "siglip_qkv", "prefix_o", "prefix_o_ragged", "prefix_down"])
def test_wide_gemm_ops(m, n, k):
    """Many-token (wide) kernel at the SigLIP / prefix shapes: 128- and 192-column tiles,
    cluster split-K on the SigLIP row epilogues, a ragged last token tile (600 tokens),
    CTA pairs with split-K 2 through the ticketed partials on the long-K prefix
    down_proj; plain, gated and in-place residual epilogues."""
    g = torch.Generator(device=DEV).manual_seed(11)
    x = _bf(torch.randn(m, k, device=DEV, generator=g))
    w = _bf(torch.randn(n, k, device=DEV, generator=g) * 0.02)
    y = (x.float() @ w.float().t()).bfloat16().float()
    _close(ops.linear(x, w), x.float() @ w.float().t())
    resid = _bf(torch.randn(m, n, device=DEV, generator=g))
    gate = torch.randn(n, device=DEV, generator=g)
    _close(ops.linear_gated_residual(x, w, resid, gate), resid.float() + y * gate.bfloat16().float(), atol=2e-2)
    r2 = resid.clone()
    ops.linear_gated_residual(x, w, r2, None, out=r2)
    _close(r2, resid.float() + y, atol=2e-2)
