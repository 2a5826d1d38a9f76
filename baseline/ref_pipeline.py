"""``sample_actions`` on the host CPU through the reference's own model code.

The reference arm of ``bench.py`` and the tests that run the reference use this
module.  It builds, from the same seeded synthetic state dict the GPU engine
loads, the models the reference runs on its hot path:

* the action expert and the PaliGemma language model as the reference's vendored
  ``GemmaModel`` (``pi05_infer/gemma/modeling_gemma.py``, loaded from
  ``baseline/_ref`` by ``ref_loader``), adaRMS for the expert, plain RMSNorm for the
  prefix LM;
* SigLIP So400m/14 as the transformers ``SiglipVisionModel`` (the reference takes
  it from transformers, ``openpi_patched/gemma_pytorch.py:106-107``) followed by
  the linear multimodal projector.

The glue between them is restated from the reference because its openpi imports
block it here: the timestep sinusoid and time MLP (``pi0_pytorch.py:29-46,
325-330``), masks and positions (``engine.py:453-491``, ``pi0_pytorch.py:56-85,
160-163``), the language embedding scale (``pi0_pytorch.py:225-228``), the
action in/out projections (``engine.py:681-768``) and the Euler update
(``engine.py:629-676``).

Test and benchmark infrastructure only; the product never imports it.
"""

from __future__ import annotations

import importlib.util
import math
import os
import sys
from typing import Dict, List, Optional, Tuple

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
if os.path.join(REPO, "pi05-infer_b200") not in sys.path:
    sys.path.insert(0, os.path.join(REPO, "pi05-infer_b200"))

from pi05_infer import synthetic  # noqa: E402
from pi05_infer.config import GEMMA_2B, GEMMA_300M, SIGLIP_SO400M, GemmaShape, SiglipShape  # noqa: E402

MASK_NEG = -2.3819763e38


def _ref_loader():
    name = "pi05_ref_loader"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(name, os.path.join(HERE, "ref_loader.py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return sys.modules[name]


def _strip(sd, prefix):
    return {k[len(prefix):]: v for k, v in sd.items() if k.startswith(prefix)}


def build_gemma(mod, sd, prefix: str, shape: GemmaShape, depth: int, adarms: bool, dtype=torch.float32,
                device="cpu"):
    """A reference ``GemmaModel`` holding the weights under ``prefix`` of ``sd``.
    Under ``dtype=torch.bfloat16`` the GEMM weights are bf16 and the norms stay fp32
    (``gemma_pytorch.py:93-104``)."""
    cfg = _ref_loader().gemma_config(shape.width, depth, shape.mlp_dim, shape.num_heads, shape.num_kv_heads,
                                     shape.head_dim, adarms=adarms)
    model = mod.GemmaModel(cfg)
    model.embed_tokens = None
    w = {k: v for k, v in _strip(sd, prefix).items() if not k.startswith("embed_tokens")}
    missing, unexpected = model.load_state_dict(w, strict=False, assign=True)
    assert not unexpected, unexpected
    assert all(k.startswith("embed_tokens") for k in missing), missing
    if dtype == torch.bfloat16:
        model.to(torch.bfloat16)
        for name, prm in model.named_parameters():
            if any(s in name for s in ("input_layernorm", "post_attention_layernorm", "norm.")):
                prm.data = prm.data.float()
    model.to(device)
    model.eval()
    return model


def time_cond(w, t: float, device="cpu") -> torch.Tensor:
    """Sinusoid with fp64 periods (``pi0_pytorch.py:29-46``) and the time MLP (``:325-330``)."""
    dim = w["time_mlp_in.weight"].shape[1]
    fraction = torch.linspace(0.0, 1.0, dim // 2, dtype=torch.float64)
    period = 4e-3 * (4.0 / 4e-3) ** fraction
    x = (1.0 / period * 2 * math.pi)[None, :] * torch.tensor([t], dtype=torch.float64)[:, None]
    emb = torch.cat([torch.sin(x), torch.cos(x)], dim=1).float().to(device)
    f = torch.nn.functional
    x = f.silu(f.linear(emb, w["time_mlp_in.weight"].to(device), w["time_mlp_in.bias"].to(device)))
    return f.silu(f.linear(x, w["time_mlp_out.weight"].to(device), w["time_mlp_out.bias"].to(device)))


def velocity(model, w, x_t, t: float, kv, prefix_pad, device="cpu", static_kv=False) -> torch.Tensor:
    """v_t ``[1, M, 32]`` for x_t ``[1, M, 32]`` over the prefix cache ``kv`` (list of
    (K, V) ``[1, 1, P, D]`` in the model's dtype).  ``static_kv`` puts the model in the
    state the reference's engine uses for the denoise loop: fused q|k|v weight built,
    static KV buffers primed (``modeling_gemma.py:312-351,605-615``)."""
    f = torch.nn.functional
    m = x_t.shape[1]
    p = prefix_pad.shape[1]
    x_t = x_t.to(device)
    emb = f.linear(x_t, w["action_in_proj.weight"].to(device), w["action_in_proj.bias"].to(device))
    cond = time_cond(w, t, device)
    suffix_pad = torch.ones(1, m, dtype=torch.bool)
    att = torch.tensor([[1] + [0] * (m - 1)])
    cums = torch.cumsum(att, dim=1)
    suffix_2d = (cums[:, None, :] <= cums[:, :, None]) & (suffix_pad[:, None, :] & suffix_pad[:, :, None])
    full = torch.cat([prefix_pad[:, None, :].expand(1, m, p), suffix_2d], dim=2)
    mask4 = torch.where(full[:, None], 0.0, MASK_NEG).to(device)
    pos = (prefix_pad.sum(-1)[:, None] + torch.cumsum(suffix_pad, dim=1) - 1).to(device)
    if static_kv:
        model.build_qkv_fused()
        model.prime_kv_static(kv, m)
    out = model(inputs_embeds=emb, attention_mask=mask4, position_ids=pos, past_key_values=list(kv), use_cache=False,
                cache_position=torch.arange(p, p + m, device=device), adarms_cond=cond).last_hidden_state
    out = out[:, -m:].to(torch.float32)
    return f.linear(out, w["action_out_proj.weight"].to(device), w["action_out_proj.bias"].to(device))


def euler(x, v, t, delta):
    """flow_ode mean of ``sample_mean_var_val`` (``engine.py:664-675``)."""
    x0 = x - v * t
    x1 = x + v * (1 - t)
    return x0 * (1 - (t - delta)) + x1 * (t - delta)


class RefCpuPipeline:
    """The reference's models on the host CPU, fp32, for one observation at a time.

    ``workload`` "e2e": SigLIP + projector over the views, the language embedding,
    the prefix LM with ``use_cache=True`` (KV cache), then the Euler loop of the
    action expert.  "denoise": the Euler loop alone over a given prefix KV cache."""

    def __init__(self, workload: str = "e2e", num_views: int = 3, prompt_len: int = 200, num_steps: int = 10,
                 expert: GemmaShape = GEMMA_300M, lm: GemmaShape = GEMMA_2B, vis: SiglipShape = SIGLIP_SO400M,
                 sd: Optional[Dict[str, torch.Tensor]] = None):
        rl = _ref_loader()
        if not rl.available():
            raise FileNotFoundError("reference not installed under baseline/_ref")
        mod = rl.load_modeling_gemma(fused_ops=None, tag="cpu_pipeline")
        self.workload = workload
        self.num_views = num_views
        self.prompt_len = prompt_len
        self.num_steps = num_steps
        self.vis = vis
        if sd is None:
            sd = {}
            sd.update(synthetic.make_expert_weights(0, expert))
            if workload == "e2e":
                sd.update(synthetic.make_prefix_lm_weights(10, lm, with_embedding=True))
                sd.update(synthetic.make_siglip_weights(20, vis))
        self.w = sd
        self.expert = build_gemma(mod, sd, synthetic.EXPERT_PREFIX, expert, expert.depth, True)
        self.lm = None
        self.siglip = None
        if workload == "e2e":
            self.lm = build_gemma(mod, sd, synthetic.LM_PREFIX, lm, lm.depth, False)
            self.siglip = self._build_siglip(sd, vis)
            self.embed = sd[synthetic.EMBED_KEY]
            self.proj_w = sd[synthetic.PROJECTOR_PREFIX + "weight"]
            self.proj_b = sd[synthetic.PROJECTOR_PREFIX + "bias"]

    @staticmethod
    def _build_siglip(sd, vis: SiglipShape):
        from transformers import SiglipVisionConfig, SiglipVisionModel

        cfg = SiglipVisionConfig(hidden_size=vis.width, intermediate_size=vis.mlp_dim, num_hidden_layers=vis.depth,
                                 num_attention_heads=vis.num_heads, image_size=vis.image_size, patch_size=vis.patch,
                                 hidden_act="gelu_pytorch_tanh", layer_norm_eps=vis.ln_eps)
        cfg._attn_implementation = "eager"
        model = SiglipVisionModel(cfg)
        w = {"vision_model." + k: v for k, v in _strip(sd, synthetic.VISION_PREFIX).items()}
        missing, unexpected = model.load_state_dict(w, strict=False, assign=True)
        assert not unexpected, unexpected
        model.eval()
        return model

    def prefix_kv(self, images: torch.Tensor, tokens: torch.Tensor, prefix_pad: torch.Tensor):
        """SigLIP + projector, scaled token embeddings, prefix LM (``use_cache=True``):
        returns the KV cache as ``[(K, V) [1, 1, P, D]]``."""
        f = torch.nn.functional
        hid = self.siglip(pixel_values=images).last_hidden_state
        feats = f.linear(hid, self.proj_w, self.proj_b).reshape(1, -1, self.proj_w.shape[0])
        lang = self.embed[tokens.long()].reshape(1, -1, self.embed.shape[1]) * math.sqrt(self.embed.shape[1])
        embs = torch.cat([feats, lang], dim=1)
        p = embs.shape[1]
        pad = prefix_pad.reshape(1, p)
        m2 = pad[:, None, :] & pad[:, :, None]
        mask4 = torch.where(m2[:, None], 0.0, MASK_NEG)
        pos = torch.cumsum(pad.long(), dim=1) - 1
        out = self.lm(inputs_embeds=embs, attention_mask=mask4, position_ids=pos, use_cache=True,
                      cache_position=torch.arange(p))
        cache = out.past_key_values
        kv = []
        for i in range(len(self.lm.layers)):
            layer = cache.layers[i] if hasattr(cache, "layers") else None
            k = layer.keys if layer is not None else cache[i][0]
            v = layer.values if layer is not None else cache[i][1]
            kv.append((k, v))
        return kv

    def denoise(self, noise: torch.Tensor, kv, prefix_pad: torch.Tensor) -> torch.Tensor:
        """The Euler loop (``engine.py:390-405``): noise ``[1, 50, 32]`` -> actions."""
        n = self.num_steps
        ts = torch.cat([torch.linspace(1, 1 / n, n), torch.zeros(1)])
        x = noise.float()
        pad = prefix_pad.reshape(1, -1)
        for s in range(n):
            v = velocity(self.expert, self.w, x, float(ts[s]), kv, pad)
            t = ts[s]
            x = euler(x, v, t, ts[s] - ts[s + 1])
        return x

    @torch.no_grad()
    def sample_actions(self, images, tokens, prefix_pad, noise, kv=None) -> torch.Tensor:
        if self.workload == "e2e":
            kv = self.prefix_kv(images, tokens, prefix_pad)
        return self.denoise(noise, kv, prefix_pad)
