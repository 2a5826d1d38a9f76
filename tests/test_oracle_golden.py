"""Pin the CPU oracle to the reference's own outputs (committed golden vectors).

The fixtures were produced by ``tests/golden/make_golden.py`` running the
reference's vendored ``GemmaModel`` (expert and prefix LM) and transformers'
SigLIP.  Tolerances: fp32 cases agree to ~1e-5 relative (summation order only);
the bf16 case agrees within bf16 rounding noise (the oracle rounds once where
the reference's eager ops round twice, e.g. ``x + y*gate``).
"""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, load_oracle

from pi05_infer import synthetic
from pi05_infer.config import GemmaShape, SiglipShape

oracle = load_oracle()


def _load(name):
    return dict(np.load(os.path.join(GOLDEN, name)))


def _cos(a, b):
    a = torch.as_tensor(a).flatten().double()
    b = torch.as_tensor(b).flatten().double()
    return float(a @ b / (a.norm() * b.norm()))


def _expert_setup(g):
    depth, p = int(g["depth"]), int(g["prefix_len"])
    shape = GemmaShape(width=1024, depth=depth, mlp_dim=4096, num_heads=8, num_kv_heads=1, head_dim=256)
    w = synthetic.make_expert_weights(0, shape)
    kv = [(k[0, 0], v[0, 0]) for k, v in synthetic.make_prefix_kv(1, depth, p)]
    noise = synthetic.make_noise(2)[0]
    pad = torch.from_numpy(g["prefix_pad"])
    return depth, w, kv, noise, pad


def test_config1_velocity_fp32():
    g = _load("expert_fp32_config1.npz")
    depth, w, kv, noise, pad = _expert_setup(g)
    table = oracle.adarms_table(w, depth, 1, synthetic.EXPERT_PREFIX)  # t = 1.0
    v = oracle.velocity(w, noise, kv, table[0], pad, depth, "fp32")
    ref = torch.from_numpy(g["velocities"][0])
    err = (v - ref).abs().max().item()
    assert err < 1e-4 * max(1.0, ref.abs().max().item()), err
    assert _cos(v, ref) > 0.999999


def test_loop_fp32_small():
    g = _load("expert_fp32_loop_small.npz")
    depth, w, kv, noise, pad = _expert_setup(g)
    vels = []
    x = oracle.denoise_loop(w, noise, kv, pad, depth, int(g["num_steps"]), "fp32", velocities=vels)
    for s, v in enumerate(vels):
        assert _cos(v, g["velocities"][s]) > 0.999999
    assert (x - torch.from_numpy(g["actions"])).abs().max().item() < 1e-4


def test_loop_bf16_small():
    g = _load("expert_bf16_small.npz")
    depth, w, kv, noise, pad = _expert_setup(g)
    kv = [(k.bfloat16().float(), v.bfloat16().float()) for k, v in kv]
    vels = []
    x = oracle.denoise_loop(w, noise, kv, pad, depth, int(g["num_steps"]), "bf16", velocities=vels)
    for s, v in enumerate(vels):
        assert _cos(v, g["velocities"][s]) > 0.9999, s
    assert (x - torch.from_numpy(g["actions"])).abs().max().item() < 2e-2


def test_prefix_kv_fp32_small():
    g = _load("prefix_fp32_small.npz")
    depth, p, width, mlp = (int(g[k]) for k in ("depth", "prefix_len", "width", "mlp"))
    shape = GemmaShape(width=width, depth=depth, mlp_dim=mlp, num_heads=8, num_kv_heads=1, head_dim=256)
    w = synthetic.make_prefix_lm_weights(10, shape)
    embs = synthetic.make_prefix_embeddings(3, p, width)[0]
    pad = torch.from_numpy(g["prefix_pad"])
    kv = oracle.prefix_lm_kv(w, embs, pad, depth, "fp32")
    valid = pad.bool()
    for i in range(depth):
        for j, name in enumerate(("k", "v")):
            got = kv[i][j][valid]
            ref = torch.from_numpy(g[name][i])[valid]
            assert (got - ref).abs().max().item() < 1e-4 * max(1.0, ref.abs().max().item()), (i, name)


def test_siglip_fp32_small():
    g = _load("siglip_fp32_small.npz")
    depth, size = int(g["depth"]), int(g["image_size"])
    shape = SiglipShape(depth=depth, image_size=size)
    w = synthetic.make_siglip_weights(20, shape)
    imgs = synthetic.make_images(4, 2, size)
    f = oracle.siglip_image_features(w, imgs, depth, "fp32")
    ref = torch.from_numpy(g["features"])
    assert (f - ref).abs().max().item() < 1e-4 * max(1.0, ref.abs().max().item())


def test_euler_is_x_minus_delta_v():
    x = torch.randn(50, 32)
    v = torch.randn(50, 32)
    out = oracle.euler(x, v, 0.7, 0.1)
    assert torch.allclose(out, x - 0.1 * v, atol=1e-5)


def test_masks():
    pad = torch.tensor([1, 1, 0, 1], dtype=torch.bool)
    m = oracle.suffix_mask(pad, 3)
    assert m.shape == (3, 7)
    assert (m[:, 2] < -1e38).all() and (m[:, [0, 1, 3, 4, 5, 6]] == 0).all()
    pm = oracle.prefix_mask(pad)
    assert pm[0, 2] < -1e38 and pm[2, 0] < -1e38 and pm[0, 3] == 0


def test_oracle_transforms_known_answers():
    """Image scaling and resize-with-pad geometry, and Normalize / Unnormalize as
    inverse pairs (oracle of the preprocessing kernels)."""
    img = torch.tensor([0, 255, 51, 204], dtype=torch.uint8).repeat(224 * 56).reshape(1, 224, 224, 1).expand(
        1, 224, 224, 3).contiguous()
    out = oracle.preprocess_images(img, 224)
    assert torch.allclose(out[0, 0, 0, :4], torch.tensor([-1.0, 1.0, -0.6, 0.6]), atol=1e-6)
    wide = torch.full((1, 480, 640, 3), 255, dtype=torch.uint8)
    out = oracle.preprocess_images(wide, 224)
    # 480 x 640 -> 168 x 224, centred: rows 28 .. 195 white, the border black
    assert torch.all(out[:, :, 28:196] == 1.0) and torch.all(out[:, :, :28] == -1.0) and torch.all(out[:, :, 196:] == -1.0)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4, 8, generator=g)
    a = torch.randn(8, generator=g)
    b = a + 2.0
    for quant in (False, True):
        y = oracle.normalize(x, a, b, quant, 32)
        assert y.shape == (4, 32) and torch.all(y[:, 8:] == 0)
        assert torch.allclose(oracle.unnormalize(y, a, b, quant, 8), x, atol=1e-5)
