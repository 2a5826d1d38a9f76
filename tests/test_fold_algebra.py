"""CPU check of the folded-norm algebra used by the GEMM epilogues.

The reference normalises, rounds the normalised activation to bf16 and projects
it (modeling_gemma.py:82-116 for the adaRMS norm, torch LayerNorm in SigLIP).  The
kernels instead fold the norm's per-column scale into a bf16 copy of the weights
and apply the per-token statistics to the fp32 accumulator:

  adaRMS:    W . bf16(h * rstd * (1 + s) + shift)  ~  rstd * (W' . h) + W . shift,
             W' = bf16(W * (1 + s))
  LayerNorm: W . bf16((h - mean) * rstd * g + b)   ~  rstd * (W' . h - mean * colsum(W')) + W . b,
             W' = bf16(W * g), colsum over the rounded W'

Both sides are computed here in fp64 from the same bf16 operands; the folded form
must agree with the reference form to within the bf16 rounding of one operand (the
tests' relative tolerance 1e-2 of the output scale).  The LayerNorm case includes a
token whose mean is 20x its spread: the column sums are taken of the rounded W', so
the mean term cancels exactly and the error stays relative to the centred values.
"""

import torch


def _bf(x):
    return x.to(torch.bfloat16).double()


def test_folded_adarms_matches_normalise_then_project():
    g = torch.Generator().manual_seed(0)
    n, k, t = 256, 1024, 50
    w = _bf(torch.randn(n, k, generator=g) * 0.02)
    h = _bf(torch.randn(t, k, generator=g))
    scale = torch.randn(k, generator=g).double() * 0.5
    shift = torch.randn(k, generator=g).double() * 0.5
    rstd = 1.0 / torch.sqrt((h * h).mean(1, keepdim=True) + 1e-6)
    ref = _bf(h * rstd * (1 + scale) + shift) @ w.T
    w_f = _bf(w * (1 + scale))
    got = rstd * (h @ w_f.T) + (w @ shift)[None]
    err = (got - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item(), err


def test_folded_layernorm_matches_normalise_then_project():
    g = torch.Generator().manual_seed(1)
    n, k, t = 256, 1152, 64
    w = _bf(torch.randn(n, k, generator=g) * 0.02)
    h = torch.randn(t, k, generator=g)
    h[0] += 20.0  # a token whose mean is 20x its spread
    h = _bf(h)
    gamma = 1 + torch.randn(k, generator=g).double() * 0.2
    beta = torch.randn(k, generator=g).double() * 0.2
    mean = h.mean(1, keepdim=True)
    # statistics as the kernels form them: per-part sums, variance E[x^2] - mean^2
    var = (h * h).mean(1, keepdim=True) - mean * mean
    rstd = 1.0 / torch.sqrt(var + 1e-6)
    ref_rstd = 1.0 / torch.sqrt(((h - mean) ** 2).mean(1, keepdim=True) + 1e-6)
    ref = _bf((h - mean) * ref_rstd * gamma + beta) @ w.T
    w_f = _bf(w * gamma)
    colsum = w_f.sum(1)
    got = rstd * (h @ w_f.T - mean * colsum[None]) + (w @ beta)[None]
    scale = ref.abs().max(1, keepdim=True).values
    assert ((got - ref).abs() <= 1e-2 * scale).all()
    # without the rounded column sums (colsum of the unrounded W * gamma) the
    # large-mean token's error grows with its mean
    bad = rstd * (h @ w_f.T - mean * (w * gamma).sum(1)[None]) + (w @ beta)[None]
    assert (bad[0] - ref[0]).abs().max() > (got[0] - ref[0]).abs().max()
