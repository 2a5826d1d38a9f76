"""GPU tests of the engine/builder API around ``sample_actions``.

* ``invalidate_weight_derived_caches`` (reference ``engine.py:526-554``): weights
  mutated in place are picked up by the already captured CUDA graph (its derived
  buffers -- fused q|k|v, folded norm copies, the adaRMS modulation table, the
  SigLIP / prefix folds -- are rebuilt at their old addresses), and the result
  matches the oracle on the new weights.
* ``build_model`` / ``get_model`` (``builder.py:34-151``) from a safetensors file
  with the reference's key names, and from an FSDP ``full_weights.pt``.
* ``sample_actions`` with ``bsize > 1`` and ``predict_action_batch``.

Reduced depth (2 SigLIP, 2 prefix, 2 expert layers, 3 Euler steps) keeps the oracle
fast; tolerances are the north-star action tolerance (max-abs <= 2e-2).
"""

import os

import pytest
import torch

from conftest import load_oracle

from pi05_infer import build_model, get_model, ops, synthetic
from pi05_infer.config import EngineConfig, GemmaShape, SiglipShape
from pi05_infer.engine import Observation, OpenPi0Inference

pytestmark = pytest.mark.gpu

oracle = load_oracle()

EXPERT = GemmaShape(width=1024, depth=2, mlp_dim=4096, num_heads=8, num_kv_heads=1, head_dim=256)
LM = GemmaShape(width=2048, depth=2, mlp_dim=16384, num_heads=8, num_kv_heads=1, head_dim=256)
VIS = SiglipShape(depth=2)


def _cfg():
    return EngineConfig(num_steps=3, expert=EXPERT, prefix_lm=LM, siglip=VIS)


def _weights(seed):
    sd = {}
    sd.update(synthetic.make_expert_weights(seed, EXPERT))
    sd.update(synthetic.make_prefix_lm_weights(seed + 10, LM, with_embedding=True))
    sd.update(synthetic.make_siglip_weights(seed + 20, VIS))
    return sd


def _observation(seed, batch=1):
    g = torch.Generator().manual_seed(seed)
    imgs = {f"cam{i}": torch.rand((batch, 3, 224, 224), generator=g) * 2 - 1 for i in range(3)}
    masks = {k: torch.ones(batch, dtype=torch.bool) for k in imgs}
    toks = torch.randint(0, synthetic.VOCAB_SIZE, (batch, 200), generator=g)
    tmask = torch.ones(batch, 200, dtype=torch.bool)
    tmask[:, 190:] = False
    return Observation(imgs, masks, toks, tmask, torch.zeros(batch, 32))


def _oracle_actions(sd, obs, noise, i=0):
    imgs = torch.cat([obs.images[k][i: i + 1] for k in obs.images], 0)
    feats = oracle.siglip_image_features(sd, imgs, VIS.depth, "bf16")
    lang = oracle.embed_language(sd[synthetic.EMBED_KEY], obs.tokenized_prompt[i], "bf16")
    embs = oracle.embed_prefix(feats, lang)
    masks = [obs.image_masks[k][i].reshape(1).expand(256) for k in obs.images]
    pad = torch.cat(masks + [obs.tokenized_prompt_mask[i]])
    kv = oracle.prefix_lm_kv(sd, embs, pad, LM.depth, "bf16")
    return oracle.denoise_loop(sd, noise, kv, pad, EXPERT.depth, 3, "bf16")


def test_weight_refresh_replays_captured_graph():
    sd = _weights(0)
    eng = OpenPi0Inference(_cfg(), sd, device="cuda")
    obs = _observation(100)
    noise = synthetic.make_noise(2)
    act0 = eng.sample_actions(obs, noise=noise)["actions"][0].cpu()
    graph = eng._graphs["full"]
    table_ptr = eng._denoise.table.data_ptr()
    # an RL weight sync: every weight of the checkpoint changes in place
    new = _weights(7)
    for k, t in sd.items():
        t.copy_(new[k])
    eng.invalidate_weight_derived_caches()
    act1 = eng.sample_actions(obs, noise=noise)["actions"][0].cpu()
    assert eng._graphs["full"] is graph, "the captured graph was replaced instead of replayed"
    assert eng._denoise.table.data_ptr() == table_ptr
    assert ops.read_device_status() == 0
    assert (act1 - act0).abs().max().item() > 1e-2  # the new weights are in use
    ref = _oracle_actions(new, obs, noise[0])
    err = (act1 - ref).abs().max().item()
    assert err <= 2e-2, err


def test_build_model_from_reference_checkpoints(tmp_path):
    from safetensors.torch import save_file

    sd = _weights(0)
    obs = _observation(100)
    noise = synthetic.make_noise(2)
    direct = OpenPi0Inference(_cfg(), sd, device="cuda").sample_actions(obs, noise=noise)["actions"].cpu()
    # safetensors with the reference's key names, split over two shards
    keys = sorted(sd)
    half = len(keys) // 2
    d1 = tmp_path / "st"
    d1.mkdir()
    save_file({k: sd[k].contiguous() for k in keys[:half]}, str(d1 / "model-00001.safetensors"))
    save_file({k: sd[k].contiguous() for k in keys[half:]}, str(d1 / "model-00002.safetensors"))
    kw = dict(num_steps=3, expert=EXPERT, prefix_lm=LM, siglip=VIS)
    eng = build_model(str(d1), "pi05_libero", **kw)
    got = eng.sample_actions(obs, noise=noise)["actions"].cpu()
    assert torch.equal(got, direct)
    # FSDP checkpoint layout: model_state_dict/full_weights.pt, through get_model
    d2 = tmp_path / "fsdp"
    os.makedirs(d2 / "model_state_dict")
    torch.save(sd, str(d2 / "model_state_dict" / "full_weights.pt"))
    cfg = {"model_path": str(d2), "openpi": {"config_name": "pi05_turtle", **kw}, "openpi_data": None}
    got2 = get_model(cfg).sample_actions(obs, noise=noise)["actions"].cpu()
    assert torch.equal(got2, direct)
    with pytest.raises(ValueError):
        build_model(str(d1), "pi0_libero")


def test_batched_observations():
    sd = _weights(0)
    eng = OpenPi0Inference(_cfg(), sd, device="cuda")
    obs = _observation(200, batch=3)
    obs.image_masks["cam1"][1] = False  # observation 1 misses a view
    noise = synthetic.make_noise(4, batch=3)
    act = eng.sample_actions(obs, noise=noise)["actions"].cpu()
    assert act.shape == (3, 50, 32)
    assert ops.read_device_status() == 0
    for i in range(3):
        ref = _oracle_actions(sd, obs, noise[i], i)
        err = (act[i] - ref).abs().max().item()
        assert err <= 2e-2, (i, err)
    # predict_action_batch: the same dict observation in; without norm statistics the
    # output transform is the policy's slice (libero: 7 action dims)
    env = {"image": obs.images, "image_mask": obs.image_masks, "tokenized_prompt": obs.tokenized_prompt,
           "tokenized_prompt_mask": obs.tokenized_prompt_mask, "state": obs.state}
    out = eng.predict_action_batch(env)
    assert out.shape == (3, 50, 7)
    with pytest.raises(ValueError):
        eng.sample_actions(obs, noise=synthetic.make_noise(4, batch=2))
