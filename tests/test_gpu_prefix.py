"""GPU parity of the prefix LM (Gemma-2B width, KV-cache fill) and the language
embedding against the CPU oracle (bf16 policy).

Tolerance: per-layer K/V cosine >= 0.9999 over valid tokens and max-abs error
within a few bf16 ulps of the values' scale.
"""

import math

import pytest
import torch

from conftest import load_oracle

from pi05_infer import ops, synthetic
from pi05_infer.config import GemmaShape
from pi05_infer.engine import OpenPi0Inference
from pi05_infer.prefix import PrefixRunner, PrefixWeights, embed_tokens

pytestmark = pytest.mark.gpu

oracle = load_oracle()


def _cos(a, b):
    a = a.flatten().double()
    b = b.flatten().double()
    return float(a @ b / (a.norm() * b.norm()))


@pytest.mark.parametrize("p,n_pad,depth", [(968, 37, 2), (300, 0, 3)])
def test_prefix_kv_parity(p, n_pad, depth):
    shape = GemmaShape(width=2048, depth=depth, mlp_dim=16384, num_heads=8, num_kv_heads=1, head_dim=256)
    sd = synthetic.make_prefix_lm_weights(10, shape)
    embs = synthetic.make_prefix_embeddings(3, p, 2048)[0]
    valid = torch.ones(p, dtype=torch.bool)
    if n_pad:
        valid[-n_pad:] = False
    w = PrefixWeights(sd, shape, "cuda")
    kc = [torch.zeros(1, p + 50, 256, dtype=torch.bfloat16, device="cuda") for _ in range(depth)]
    vc = [torch.zeros(1, p + 50, 256, dtype=torch.bfloat16, device="cuda") for _ in range(depth)]
    r = PrefixRunner(w, p, kc, vc)
    r.run(embs.cuda(), valid.cuda())
    assert ops.read_device_status() == 0
    ref = oracle.prefix_lm_kv(sd, embs.bfloat16().float(), valid, depth, "bf16")
    for i in range(depth):
        for j, cache in enumerate((kc, vc)):
            got = cache[i][0, :p].float().cpu()[valid]
            exp = ref[i][j][valid]
            c = _cos(got, exp)
            assert c >= 0.9999, (i, j, c)
            scale = exp.abs().max().item()
            assert (got - exp).abs().max().item() <= 0.05 * scale, (i, j)
        assert cache[i][0, p:].abs().sum().item() == 0  # suffix rows untouched


def test_prefix_folded_norm_matches_norm_kernels():
    # The folded RMSNorms (weights carry (1 + w); q|k|v and gate/up scale each token
    # by its rstd from the residual GEMMs' row statistics) against the same layers
    # with the RMSNorm kernels: per-layer K/V within the prefix tolerance.
    p, depth = 968, 3
    shape = GemmaShape(width=2048, depth=depth, mlp_dim=16384, num_heads=8, num_kv_heads=1, head_dim=256)
    sd = synthetic.make_prefix_lm_weights(10, shape)
    embs = synthetic.make_prefix_embeddings(3, p, 2048)[0].cuda()
    valid = torch.ones(p, dtype=torch.bool, device="cuda")
    valid[-20:] = False
    w = PrefixWeights(sd, shape, "cuda")
    assert w.fold
    caches = []
    for folded in (True, False):
        kc = [torch.zeros(1, p + 50, 256, dtype=torch.bfloat16, device="cuda") for _ in range(depth)]
        vc = [torch.zeros(1, p + 50, 256, dtype=torch.bfloat16, device="cuda") for _ in range(depth)]
        r = PrefixRunner(w, p, kc, vc)
        if not folded:
            r.plan.row_stats = None
        r.run(embs, valid)
        caches.append((kc, vc))
    assert ops.read_device_status() == 0
    vm = valid.cpu()
    for i in range(depth):
        for j in range(2):
            a = caches[0][j][i][0, :p].float().cpu()[vm]
            b = caches[1][j][i][0, :p].float().cpu()[vm]
            assert _cos(a, b) >= 0.9999, (i, j)
            assert (a - b).abs().max().item() <= 0.05 * b.abs().max().item(), (i, j)


def test_embed_tokens():
    g = torch.Generator(device="cuda").manual_seed(7)
    table = (torch.randn(1000, 2048, device="cuda", generator=g) * 0.02).bfloat16()
    ids = torch.randint(0, 1000, (200,), device="cuda", generator=g, dtype=torch.int32)
    out = torch.empty(200, 2048, dtype=torch.bfloat16, device="cuda")
    ws = ops.workspace(out.device)
    embed_tokens(table, ids, out, math.sqrt(2048), ws, torch.cuda.current_stream().cuda_stream)
    ref = oracle.embed_language(table.float().cpu(), ids.cpu(), "bf16")
    assert torch.equal(out.float().cpu(), ref)
    assert ops.read_device_status() == 0
    # out-of-range id: zero row + status bit, no fault
    ids[3] = 5000
    embed_tokens(table, ids, out, math.sqrt(2048), ws, torch.cuda.current_stream().cuda_stream)
    assert out[3].abs().sum().item() == 0
    assert ops.read_device_status() == 0x20


def test_engine_config2_pipeline_runs():
    """Prefix LM from N(0,1) embeddings -> KV -> 10-step loop, through the engine API."""
    eng = OpenPi0Inference.synthetic(device="cuda", seed=0)
    eng.prepare(None)
    a1 = eng.denoise(synthetic.make_noise(2))["actions"]
    a2 = eng.denoise(synthetic.make_noise(2).pin_memory())["actions"]
    assert a1.shape == (1, 50, 32) and torch.isfinite(a1).all()
    assert torch.equal(a1, a2)  # deterministic replays
    assert ops.read_device_status() == 0
