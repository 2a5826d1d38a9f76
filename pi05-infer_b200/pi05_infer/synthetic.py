"""Seeded synthetic weights and inputs (no checkpoint or dataset is available).

Every tensor is drawn N(0, 0.02) in a fixed key order from one ``torch.Generator``
so that the CPU oracle, the golden-vector script and the GPU engine see identical
values for the same seed (torch's CPU generator is platform independent).  Key
names are the reference's ``state_dict`` names (``PI0Pytorch`` owns
``action_in_proj``/``action_out_proj``/``time_mlp_*``, ``pi0_pytorch.py:104-109``;
the expert lives under ``paligemma_with_expert.gemma_expert.model``,
``gemma_pytorch.py:78-79``), so ``build_model`` can load either these tensors or
a real checkpoint's.

Unlike the reference, which zero-inits the adaRMS ``dense``
(``modeling_gemma.py:77``), the synthetic expert draws it N(0, 0.02) too, so the
modulation path carries signal in tests.
"""

from __future__ import annotations

from collections import OrderedDict

import torch

from .config import ACTION_DIM, GEMMA_2B, GEMMA_300M, SIGLIP_SO400M, VOCAB_SIZE, GemmaShape, SiglipShape

EXPERT_PREFIX = "paligemma_with_expert.gemma_expert.model."
LM_PREFIX = "paligemma_with_expert.paligemma.model.language_model."
VISION_PREFIX = "paligemma_with_expert.paligemma.model.vision_tower.vision_model."
PROJECTOR_PREFIX = "paligemma_with_expert.paligemma.model.multi_modal_projector.linear."
EMBED_KEY = LM_PREFIX + "embed_tokens.weight"

STD = 0.02


def expert_param_shapes(shape: GemmaShape = GEMMA_300M) -> "OrderedDict[str, tuple]":
    d, f, hd = shape.width, shape.mlp_dim, shape.head_dim
    out = OrderedDict()
    for i in range(shape.depth):
        p = f"{EXPERT_PREFIX}layers.{i}."
        out[p + "self_attn.q_proj.weight"] = (shape.num_heads * hd, d)
        out[p + "self_attn.k_proj.weight"] = (shape.num_kv_heads * hd, d)
        out[p + "self_attn.v_proj.weight"] = (shape.num_kv_heads * hd, d)
        out[p + "self_attn.o_proj.weight"] = (d, shape.num_heads * hd)
        out[p + "mlp.gate_proj.weight"] = (f, d)
        out[p + "mlp.up_proj.weight"] = (f, d)
        out[p + "mlp.down_proj.weight"] = (d, f)
        out[p + "input_layernorm.dense.weight"] = (3 * d, d)
        out[p + "input_layernorm.dense.bias"] = (3 * d,)
        out[p + "post_attention_layernorm.dense.weight"] = (3 * d, d)
        out[p + "post_attention_layernorm.dense.bias"] = (3 * d,)
    out[EXPERT_PREFIX + "norm.dense.weight"] = (3 * d, d)
    out[EXPERT_PREFIX + "norm.dense.bias"] = (3 * d,)
    out["action_in_proj.weight"] = (d, ACTION_DIM)
    out["action_in_proj.bias"] = (d,)
    out["action_out_proj.weight"] = (ACTION_DIM, d)
    out["action_out_proj.bias"] = (ACTION_DIM,)
    out["time_mlp_in.weight"] = (d, d)
    out["time_mlp_in.bias"] = (d,)
    out["time_mlp_out.weight"] = (d, d)
    out["time_mlp_out.bias"] = (d,)
    return out


def prefix_lm_param_shapes(shape: GemmaShape = GEMMA_2B, with_embedding: bool = False) -> "OrderedDict[str, tuple]":
    d, f, hd = shape.width, shape.mlp_dim, shape.head_dim
    out = OrderedDict()
    for i in range(shape.depth):
        p = f"{LM_PREFIX}layers.{i}."
        out[p + "self_attn.q_proj.weight"] = (shape.num_heads * hd, d)
        out[p + "self_attn.k_proj.weight"] = (shape.num_kv_heads * hd, d)
        out[p + "self_attn.v_proj.weight"] = (shape.num_kv_heads * hd, d)
        out[p + "self_attn.o_proj.weight"] = (d, shape.num_heads * hd)
        out[p + "mlp.gate_proj.weight"] = (f, d)
        out[p + "mlp.up_proj.weight"] = (f, d)
        out[p + "mlp.down_proj.weight"] = (d, f)
        out[p + "input_layernorm.weight"] = (d,)
        out[p + "post_attention_layernorm.weight"] = (d,)
    out[LM_PREFIX + "norm.weight"] = (d,)
    if with_embedding:
        out[EMBED_KEY] = (VOCAB_SIZE, d)
    return out


def siglip_param_shapes(shape: SiglipShape = SIGLIP_SO400M) -> "OrderedDict[str, tuple]":
    w, f = shape.width, shape.mlp_dim
    out = OrderedDict()
    out[VISION_PREFIX + "embeddings.patch_embedding.weight"] = (w, 3, shape.patch, shape.patch)
    out[VISION_PREFIX + "embeddings.patch_embedding.bias"] = (w,)
    out[VISION_PREFIX + "embeddings.position_embedding.weight"] = (shape.num_patches, w)
    for i in range(shape.depth):
        p = f"{VISION_PREFIX}encoder.layers.{i}."
        for n in ("q_proj", "k_proj", "v_proj", "out_proj"):
            out[p + f"self_attn.{n}.weight"] = (w, w)
            out[p + f"self_attn.{n}.bias"] = (w,)
        out[p + "layer_norm1.weight"] = (w,)
        out[p + "layer_norm1.bias"] = (w,)
        out[p + "mlp.fc1.weight"] = (f, w)
        out[p + "mlp.fc1.bias"] = (f,)
        out[p + "mlp.fc2.weight"] = (w, f)
        out[p + "mlp.fc2.bias"] = (w,)
        out[p + "layer_norm2.weight"] = (w,)
        out[p + "layer_norm2.bias"] = (w,)
    out[VISION_PREFIX + "post_layernorm.weight"] = (w,)
    out[VISION_PREFIX + "post_layernorm.bias"] = (w,)
    out[PROJECTOR_PREFIX + "weight"] = (shape.proj_dim, w)
    out[PROJECTOR_PREFIX + "bias"] = (shape.proj_dim,)
    return out


def _draw(shapes, seed: int, device="cpu", std: float = STD) -> "OrderedDict[str, torch.Tensor]":
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = OrderedDict()
    for k, s in shapes.items():
        out[k] = torch.randn(s, generator=g, dtype=torch.float32, device=device) * std
    return out


def make_expert_weights(seed: int = 0, shape: GemmaShape = GEMMA_300M, device="cpu"):
    """Action expert + glue (config 1/2 weights), all fp32 N(0, 0.02)."""
    return _draw(expert_param_shapes(shape), seed, device)


def make_prefix_lm_weights(seed: int = 10, shape: GemmaShape = GEMMA_2B, device="cpu", with_embedding=False):
    return _draw(prefix_lm_param_shapes(shape, with_embedding), seed, device)


def make_siglip_weights(seed: int = 20, shape: SiglipShape = SIGLIP_SO400M, device="cpu"):
    return _draw(siglip_param_shapes(shape), seed, device)


def make_prefix_kv(seed: int, depth: int, prefix_len: int, head_dim: int = 256, num_kv_heads: int = 1, device="cpu"):
    """Config-1 synthetic prefix cache: ``[depth][2]`` tensors ``[1, Hkv, P, D]`` N(0, 1)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    kv = []
    for _ in range(depth):
        k = torch.randn((1, num_kv_heads, prefix_len, head_dim), generator=g, device=device)
        v = torch.randn((1, num_kv_heads, prefix_len, head_dim), generator=g, device=device)
        kv.append((k, v))
    return kv


def make_noise(seed: int = 2, batch: int = 1, horizon: int = 50, action_dim: int = ACTION_DIM, device="cpu"):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randn((batch, horizon, action_dim), generator=g, device=device)


def make_prefix_embeddings(seed: int = 3, prefix_len: int = 968, width: int = 2048, device="cpu"):
    """Config-2 synthetic prefix embeddings ``[1, P, width]`` N(0, 1)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randn((1, prefix_len, width), generator=g, device=device)


def make_images(seed: int = 4, num_views: int = 3, size: int = 224, device="cpu"):
    """Config-3 camera images ``[views, 3, size, size]`` uniform in [-1, 1]."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.rand((num_views, 3, size, size), generator=g, device=device) * 2.0 - 1.0


def make_tokens(seed: int = 5, n: int = 200, vocab: int = VOCAB_SIZE, device="cpu"):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randint(0, vocab, (1, n), generator=g, device=device)
