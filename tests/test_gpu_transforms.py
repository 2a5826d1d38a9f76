"""GPU parity of the observation preprocessing and the action output transform
(``pi05_preprocess_images``, ``pi05_normalize_rows``, ``pi05_unnormalize_rows``)
against the CPU oracle, and of ``predict_action_batch`` on environment
observations against ``sample_actions`` on the oracle-preprocessed observation.

Tolerances: images 1e-5 absolute (the kernel interpolates in pixel units and scales
afterwards; the oracle scales after torch's interpolation: fp32 rounding only);
normalisation 1e-5 relative; predict_action_batch vs the manual pipeline 5e-3
(the same bf16 pipeline on inputs that differ by fp32 rounding).
"""

import pytest
import torch

from conftest import load_oracle

from pi05_infer import ops, synthetic, transforms
from pi05_infer.config import EngineConfig, GemmaShape, SiglipShape
from pi05_infer.engine import Observation, OpenPi0Inference

pytestmark = pytest.mark.gpu

oracle = load_oracle()


@pytest.mark.parametrize("shape,chw", [((2, 224, 224), False), ((2, 480, 640), False), ((1, 256, 256), True),
                                       ((3, 100, 300), False), ((1, 640, 480), False)],
                         ids=["224", "480x640", "256-chw", "100x300", "640x480"])
def test_preprocess_images(shape, chw):
    g = torch.Generator().manual_seed(1)
    n, h, w = shape
    img = torch.randint(0, 256, (n, 3, h, w) if chw else (n, h, w, 3), generator=g, dtype=torch.uint8)
    got = transforms.preprocess_images(img.cuda(), 224).cpu()
    ref = oracle.preprocess_images(img, 224)
    assert got.shape == (n, 3, 224, 224)
    assert (got - ref).abs().max().item() <= 1e-5
    if (h, w) == (224, 224):
        assert torch.equal(got, img.permute(0, 3, 1, 2).float() / 255.0 * 2.0 - 1.0)


@pytest.mark.parametrize("quant", [False, True], ids=["mean_std", "quantiles"])
def test_normalize_unnormalize(quant):
    g = torch.Generator().manual_seed(2)
    state = torch.randn(5, 8, generator=g) * 3
    a = torch.randn(8, generator=g)
    b = a.abs() + torch.rand(8, generator=g) + 0.5 if not quant else a + torch.rand(8, generator=g) * 4 + 0.1
    stats = transforms.NormStats(mean=a, std=b, q01=a, q99=b)
    got = transforms.normalize_state(state.cuda(), stats, quant, 32).cpu()
    ref = oracle.normalize(state, a, b, quant, 32)
    assert got.shape == (5, 32) and torch.allclose(got, ref, rtol=1e-5, atol=1e-6)
    acts = torch.randn(5, 50, 32, generator=g)
    got = transforms.unnormalize_actions(acts.cuda(), stats, quant, 7).cpu()
    ref = oracle.unnormalize(acts, a, b, quant, 7)
    assert got.shape == (5, 50, 7) and torch.allclose(got, ref, rtol=1e-5, atol=1e-6)
    # no statistics: pass-through and slice / pad
    assert torch.equal(transforms.unnormalize_actions(acts.cuda(), None, quant, 6).cpu(), acts[..., :6])


def test_predict_action_batch_env_observation():
    expert = GemmaShape(width=1024, depth=2, mlp_dim=4096, num_heads=8, num_kv_heads=1, head_dim=256)
    lm = GemmaShape(width=2048, depth=2, mlp_dim=16384, num_heads=8, num_kv_heads=1, head_dim=256)
    vis = SiglipShape(depth=2)
    cfg = EngineConfig(num_steps=3, expert=expert, prefix_lm=lm, siglip=vis, policy="libero")
    sd = {}
    sd.update(synthetic.make_expert_weights(0, expert))
    sd.update(synthetic.make_prefix_lm_weights(10, lm, with_embedding=True))
    sd.update(synthetic.make_siglip_weights(20, vis))
    eng = OpenPi0Inference(cfg, sd, device="cuda")
    g = torch.Generator().manual_seed(3)
    b = 2
    env = {
        "main_images": torch.randint(0, 256, (b, 480, 640, 3), generator=g, dtype=torch.uint8),
        "wrist_images": torch.randint(0, 256, (b, 224, 224, 3), generator=g, dtype=torch.uint8),
        "extra_view_images": None,
        "states": torch.randn(b, 8, generator=g),
        "tokenized_prompt": torch.randint(0, synthetic.VOCAB_SIZE, (b, 200), generator=g),
        "tokenized_prompt_mask": torch.ones(b, 200, dtype=torch.bool),
    }
    q01 = torch.randn(32, generator=g) - 2
    q99 = q01 + 4
    stats = {"state": transforms.NormStats(torch.zeros(8), torch.ones(8), q01[:8], q99[:8]),
             "actions": transforms.NormStats(torch.zeros(7), torch.ones(7), q01[:7], q99[:7])}
    eng.set_norm_stats(stats, use_quantiles=True)
    torch.cuda.manual_seed(5)
    got = eng.predict_action_batch(env).cpu()
    assert got.shape == (b, 50, 7)
    assert ops.read_device_status() == 0
    # the same pipeline by hand: oracle preprocessing, sample_actions, oracle output transform
    imgs = {"base_0_rgb": oracle.preprocess_images(env["main_images"]).cuda(),
            "left_wrist_0_rgb": oracle.preprocess_images(env["wrist_images"]).cuda(),
            "right_wrist_0_rgb": torch.full((b, 3, 224, 224), -1.0, device="cuda")}
    masks = {"base_0_rgb": torch.ones(b, dtype=torch.bool), "left_wrist_0_rgb": torch.ones(b, dtype=torch.bool),
             "right_wrist_0_rgb": torch.zeros(b, dtype=torch.bool)}
    state = oracle.normalize(env["states"], q01[:8], q99[:8], True, 32)
    obs = Observation(imgs, masks, env["tokenized_prompt"], env["tokenized_prompt_mask"], state)
    torch.cuda.manual_seed(5)
    act = eng.sample_actions(obs)["actions"].cpu()
    ref = oracle.unnormalize(act, q01[:7], q99[:7], True, 7)
    assert (got - ref).abs().max().item() <= 5e-3
