"""Generate the golden vectors under ``tests/golden/`` from the reference itself.

Run in the build container (needs the reference tree; the GPU box never runs
this):

    python tests/golden/make_golden.py --ref <path to pi05-infer checkout>

The reference's ``pi05_infer`` package cannot be imported as a whole (it needs
openpi and transformers 4.53.2).  Its vendored action-expert module
``pi05_infer/gemma/modeling_gemma.py`` does load under the installed
transformers with two shims (``LossKwargs`` and the ``"default"`` RoPE init),
and it is that module -- the reference's own ``GemmaModel`` -- that produces the
expert and prefix-LM outputs stored here.  The glue around it (timestep MLP,
action in/out projections, Euler update) is written out below directly from
``engine.py``/``pi0_pytorch.py`` with ``torch.nn.functional`` calls.

SigLIP is not in the reference tree (it comes from transformers); its fixture is
produced by the transformers ``SiglipVisionModel`` installed here.

Seeds follow the config-1 recipe: weights seed 0, prefix KV seed 1, noise seed 2.
"""

from __future__ import annotations

import argparse
import importlib.util
import math
import os
import sys
import types
import typing

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "pi05-infer_b200"))

from pi05_infer import synthetic  # noqa: E402
from pi05_infer.config import GemmaShape  # noqa: E402


def load_reference_gemma(ref_root: str):
    import transformers.utils as tu
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS

    if not hasattr(tu, "LossKwargs"):
        class LossKwargs(typing.TypedDict, total=False):
            pass

        tu.LossKwargs = LossKwargs

    def _default_rope(config, device=None, *args, **kwargs):
        base = getattr(config, "rope_theta", None) or 10000.0
        dim = config.head_dim
        inv = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.int64).float() / dim))
        return inv, 1.0

    ROPE_INIT_FUNCTIONS["default"] = _default_rope
    pkg = types.ModuleType("_pi05_ref")
    pkg.__path__ = []
    sys.modules["_pi05_ref"] = pkg
    path = os.path.join(ref_root, "pi05_infer", "gemma", "modeling_gemma.py")
    spec = importlib.util.spec_from_file_location("_pi05_ref.modeling_gemma", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["_pi05_ref.modeling_gemma"] = mod
    spec.loader.exec_module(mod)
    return mod


def gemma_config(shape: GemmaShape, depth: int, adarms: bool):
    from transformers.models.gemma.configuration_gemma import GemmaConfig

    cfg = GemmaConfig(
        head_dim=shape.head_dim,
        hidden_size=shape.width,
        intermediate_size=shape.mlp_dim,
        num_attention_heads=shape.num_heads,
        num_hidden_layers=depth,
        num_key_value_heads=shape.num_kv_heads,
        vocab_size=8,
        hidden_activation="gelu_pytorch_tanh",
        use_adarms=adarms,
        adarms_cond_dim=shape.width if adarms else None,
    )
    cfg._attn_implementation = "eager"
    return cfg


def strip(w, prefix):
    return {k[len(prefix):]: v for k, v in w.items() if k.startswith(prefix)}


def time_cond(w, t):
    """pi0_pytorch.py:29-46 (sinusoid, fp64) and :325-330 (time MLP)."""
    dim = w["time_mlp_in.weight"].shape[1]
    fraction = torch.linspace(0.0, 1.0, dim // 2, dtype=torch.float64)
    period = 4e-3 * (4.0 / 4e-3) ** fraction
    x = (1.0 / period * 2 * math.pi)[None, :] * t.double()[:, None]
    emb = torch.cat([torch.sin(x), torch.cos(x)], dim=1).float()
    x = torch.nn.functional.silu(torch.nn.functional.linear(emb, w["time_mlp_in.weight"], w["time_mlp_in.bias"]))
    return torch.nn.functional.silu(torch.nn.functional.linear(x, w["time_mlp_out.weight"], w["time_mlp_out.bias"]))


def ref_velocity(ref, model, w, x_t, t, kv, prefix_pad, dtype):
    """engine.py:681-768 around the reference GemmaModel."""
    m = x_t.shape[1]
    p = prefix_pad.shape[1]
    emb = torch.nn.functional.linear(x_t, w["action_in_proj.weight"], w["action_in_proj.bias"])
    cond = time_cond(w, torch.tensor([t]))
    # engine.py:471-478 masks / positions; pi0_pytorch.py:56-85,160-163
    suffix_pad = torch.ones(1, m, dtype=torch.bool)
    att = torch.tensor([[1] + [0] * (m - 1)])
    cums = torch.cumsum(att, dim=1)
    suffix_2d = (cums[:, None, :] <= cums[:, :, None]) & (suffix_pad[:, None, :] & suffix_pad[:, :, None])
    full = torch.cat([prefix_pad[:, None, :].expand(1, m, p), suffix_2d], dim=2)
    mask4 = torch.where(full[:, None], 0.0, -2.3819763e38)
    pos = prefix_pad.sum(-1)[:, None] + torch.cumsum(suffix_pad, dim=1) - 1
    out = model(
        inputs_embeds=emb,
        attention_mask=mask4,
        position_ids=pos,
        past_key_values=[(k.to(dtype), v.to(dtype)) for k, v in kv],
        use_cache=False,
        cache_position=torch.arange(p, p + m),
        adarms_cond=cond,
    ).last_hidden_state
    out = out[:, -m:].to(torch.float32)
    return torch.nn.functional.linear(out, w["action_out_proj.weight"], w["action_out_proj.bias"])


def build_expert(ref, w, shape, depth, dtype):
    model = ref.GemmaModel(gemma_config(shape, depth, True))
    model.embed_tokens = None
    sd = strip(w, synthetic.EXPERT_PREFIX)
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert all(k.startswith("embed_tokens") for k in missing), missing
    if dtype == torch.bfloat16:
        model.to(torch.bfloat16)
        for name, prm in model.named_parameters():  # gemma_pytorch.py:93-104
            if any(s in name for s in ("input_layernorm", "post_attention_layernorm", "norm.")):
                prm.data = prm.data.float()
    model.eval()
    return model


def expert_case(ref, depth, prefix_len, dtype, steps):
    shape = GemmaShape(width=1024, depth=depth, mlp_dim=4096, num_heads=8, num_kv_heads=1, head_dim=256)
    w = synthetic.make_expert_weights(0, shape)
    kv = synthetic.make_prefix_kv(1, depth, prefix_len)
    noise = synthetic.make_noise(2)
    prefix_pad = torch.ones(1, prefix_len, dtype=torch.bool)
    if prefix_len >= 16:
        prefix_pad[:, prefix_len - 5 :] = False  # ragged prompt: last 5 tokens are padding
    model = build_expert(ref, w, shape, depth, dtype)
    ts = torch.cat([torch.linspace(1, 1 / steps, steps), torch.zeros(1)]) if steps else None
    x = noise
    vels = []
    with torch.no_grad():
        if steps == 0:
            vels.append(ref_velocity(ref, model, w, x, 1.0, kv, prefix_pad, dtype))
        for s in range(steps):
            v = ref_velocity(ref, model, w, x, float(ts[s]), kv, prefix_pad, dtype)
            vels.append(v)
            t = ts[s]
            d = ts[s] - ts[s + 1]
            x = (x - v * t) * (1 - (t - d)) + (x + v * (1 - t)) * (t - d)  # engine.py:664-675
    out = {
        "depth": np.int64(depth),
        "prefix_len": np.int64(prefix_len),
        "prefix_pad": prefix_pad[0].numpy(),
        "velocities": torch.stack([v[0] for v in vels]).numpy(),
    }
    if steps:
        out["actions"] = x[0].numpy()
        out["num_steps"] = np.int64(steps)
    return out


def prefix_case(ref, depth, prefix_len, width, mlp):
    shape = GemmaShape(width=width, depth=depth, mlp_dim=mlp, num_heads=8, num_kv_heads=1, head_dim=256)
    w = synthetic.make_prefix_lm_weights(10, shape)
    embs = synthetic.make_prefix_embeddings(3, prefix_len, width)
    pad = torch.ones(1, prefix_len, dtype=torch.bool)
    pad[:, prefix_len - 3 :] = False
    model = ref.GemmaModel(gemma_config(shape, depth, False))
    model.embed_tokens = None
    sd = strip(w, synthetic.LM_PREFIX)
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    model.eval()
    att = torch.zeros(1, prefix_len, dtype=torch.long)
    cums = torch.cumsum(att, dim=1)
    m2 = (cums[:, None, :] <= cums[:, :, None]) & (pad[:, None, :] & pad[:, :, None])
    mask4 = torch.where(m2[:, None], 0.0, -2.3819763e38)
    pos = torch.cumsum(pad.long(), dim=1) - 1
    with torch.no_grad():
        out = model(inputs_embeds=embs, attention_mask=mask4, position_ids=pos, use_cache=True,
                    cache_position=torch.arange(prefix_len))
    cache = out.past_key_values
    ks, vs = [], []
    for i in range(depth):
        layer = cache.layers[i] if hasattr(cache, "layers") else None
        k = layer.keys if layer is not None else cache[i][0]
        v = layer.values if layer is not None else cache[i][1]
        ks.append(k[0, 0].numpy())
        vs.append(v[0, 0].numpy())
    return {"depth": np.int64(depth), "prefix_len": np.int64(prefix_len), "width": np.int64(width),
            "mlp": np.int64(mlp), "prefix_pad": pad[0].numpy(), "k": np.stack(ks), "v": np.stack(vs)}


def siglip_case(depth, image_size):
    from transformers import SiglipVisionConfig, SiglipVisionModel

    from pi05_infer.config import SiglipShape

    shape = SiglipShape(depth=depth, image_size=image_size)
    cfg = SiglipVisionConfig(hidden_size=shape.width, intermediate_size=shape.mlp_dim, num_hidden_layers=depth,
                             num_attention_heads=shape.num_heads, image_size=image_size, patch_size=shape.patch,
                             hidden_act="gelu_pytorch_tanh", layer_norm_eps=shape.ln_eps)
    cfg._attn_implementation = "eager"
    w = synthetic.make_siglip_weights(20, shape)
    model = SiglipVisionModel(cfg)
    sd = {"vision_model." + k[len(synthetic.VISION_PREFIX):]: v for k, v in w.items() if k.startswith(synthetic.VISION_PREFIX)}
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert all("head" in k for k in missing), missing
    model.eval()
    imgs = synthetic.make_images(4, 2, image_size)
    with torch.no_grad():
        hid = model(pixel_values=imgs).last_hidden_state
        feats = torch.nn.functional.linear(hid, w[synthetic.PROJECTOR_PREFIX + "weight"], w[synthetic.PROJECTOR_PREFIX + "bias"])
    return {"depth": np.int64(depth), "image_size": np.int64(image_size), "features": feats.numpy()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("PI05_REFERENCE_ROOT", ""))
    args = ap.parse_args()
    if not args.ref or not os.path.isdir(args.ref):
        raise SystemExit("--ref must point at the reference checkout")
    torch.manual_seed(0)
    ref = load_reference_gemma(args.ref)
    cases = {
        # config 1: full 18-layer expert, fp32, P=968, one velocity at t=1.0
        "expert_fp32_config1.npz": lambda: expert_case(ref, 18, 968, torch.float32, 0),
        # reference dtype policy (bf16 GEMMs, fp32 norms) on a small case, 3 Euler steps
        "expert_bf16_small.npz": lambda: expert_case(ref, 2, 64, torch.bfloat16, 3),
        # fp32 loop on a small case: pins the Euler/table glue over several steps
        "expert_fp32_loop_small.npz": lambda: expert_case(ref, 2, 40, torch.float32, 4),
        # prefix LM (Gemma-2B width/MLP, 2 layers) KV fill with a ragged pad mask
        "prefix_fp32_small.npz": lambda: prefix_case(ref, 2, 24, 2048, 16384),
        # SigLIP tower (2 layers, 56x56 images -> 16 patches) + projector
        "siglip_fp32_small.npz": lambda: siglip_case(2, 56),
    }
    for name, fn in cases.items():
        out = fn()
        np.savez_compressed(os.path.join(HERE, name), **out)
        print("wrote", name, {k: getattr(v, "shape", v) for k, v in out.items()})


if __name__ == "__main__":
    main()
