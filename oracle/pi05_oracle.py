"""CPU oracle for pi0.5 ``sample_actions`` -- TEST INFRASTRUCTURE, NOT THE PRODUCT.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline`` /
``--impl reference`` legs may import this module, and only as the checker (or as
the timed CPU stand-in for the reference).  The engine in ``pi05-infer_b200``
never imports it and has no CPU fallback.

It restates, in plain torch on the CPU, the math the reference runs on its hot
path.  Two numeric policies:

* ``"fp32"``: everything in fp32 (config 1).
* ``"bf16"``: fp32 arithmetic with bf16 rounding at the points where the
  reference materialises a bf16 tensor (bf16 GEMM outputs, norm outputs, the
  softmax probabilities, residual stream).  Norm math, softmax, the adaRMS table,
  action in/out projections and the Euler update stay fp32 exactly as the
  reference's dtype policy keeps them (``gemma_pytorch.py:84-104``).

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own vendored
``GemmaModel`` (``pi05_infer/gemma/modeling_gemma.py``) on seeded weights and the
committed fixtures hold its outputs; ``tests/test_oracle_golden.py`` checks this
restatement against them.  The SigLIP tower and projector are third-party
(transformers 4.53.2 + openpi ``transformers_replace``, not under the reference
tree) and are pinned against the transformers SigLIP installed here instead.
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import torch

Tensor = torch.Tensor

MASK_NEG = -2.3819763e38  # pi0_pytorch.py:160-163


def _r(x: Tensor, policy: str) -> Tensor:
    """Round through bf16 under the bf16 policy (value stays an fp32 tensor)."""
    if policy == "bf16":
        return x.to(torch.bfloat16).to(torch.float32)
    return x


def _mm(a: Tensor, w: Tensor, policy: str) -> Tensor:
    """``a @ w.T`` with fp32 accumulation.  Under bf16 the weight is the bf16 copy the
    reference holds (``gemma_pytorch.py:84-104``) and the output is rounded like a
    bf16 GEMM's."""
    return _r(a.float() @ _r(w.float(), policy).t(), policy)


def gelu_tanh(x: Tensor) -> Tensor:
    """tanh-approximated GELU (``gelu_pytorch_tanh``; ``rlinf_fused_denoise.py:166-172``)."""
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)))


# ---------------------------------------------------------------------------
# timestep conditioning + adaRMS table
# ---------------------------------------------------------------------------


def sinusoid(t: Tensor, dim: int = 1024, min_period: float = 4e-3, max_period: float = 4.0) -> Tensor:
    """``create_sinusoidal_pos_embedding`` (``pi0_pytorch.py:29-46``): fp64 math, fp32 out."""
    fraction = torch.linspace(0.0, 1.0, dim // 2, dtype=torch.float64)
    period = min_period * (max_period / min_period) ** fraction
    scaling = 1.0 / period * 2 * math.pi
    x = scaling[None, :] * t.double()[:, None]
    return torch.cat([torch.sin(x), torch.cos(x)], dim=1).float()


def timesteps(num_steps: int) -> Tensor:
    """Euler schedule ``[1, ..., 1/N, 0]`` (``engine.py:411-429``)."""
    ts = torch.linspace(1, 1 / num_steps, num_steps)
    return torch.cat([ts, torch.zeros(1)])


def time_cond(w: Dict[str, Tensor], t: Tensor) -> Tensor:
    """pi0.5 time MLP (``pi0_pytorch.py:295-335``): silu(out(silu(in(sinusoid(t)))))."""
    emb = sinusoid(t, w["time_mlp_in.weight"].shape[1])
    x = torch.nn.functional.silu(emb @ w["time_mlp_in.weight"].t() + w["time_mlp_in.bias"])
    x = x @ w["time_mlp_out.weight"].t() + w["time_mlp_out.bias"]
    return torch.nn.functional.silu(x)


def adarms_norm_keys(prefix: str, depth: int) -> List[str]:
    keys = []
    for i in range(depth):
        keys.append(f"{prefix}layers.{i}.input_layernorm.dense")
        keys.append(f"{prefix}layers.{i}.post_attention_layernorm.dense")
    keys.append(f"{prefix}norm.dense")
    return keys


def adarms_table(w: Dict[str, Tensor], depth: int, num_steps: int, prefix: str) -> Tensor:
    """``_compute_adarms_table`` (``engine.py:578-599``): ``[num_steps, n_norm, 3*width]`` fp32."""
    ts = timesteps(num_steps)
    rows = []
    for s in range(num_steps):
        cond = time_cond(w, ts[s : s + 1])  # [1, width]
        mods = [cond @ w[k + ".weight"].t() + w[k + ".bias"] for k in adarms_norm_keys(prefix, depth)]
        rows.append(torch.cat(mods, dim=0))  # [n_norm, 3*width]
    return torch.stack(rows, 0)


# ---------------------------------------------------------------------------
# norms, RoPE, attention
# ---------------------------------------------------------------------------


def ada_rms_norm(x: Tensor, mod: Tensor, eps: float, policy: str) -> Tuple[Tensor, Tensor]:
    """adaRMS (``modeling_gemma.py:82-116``): fp32 stats, ``n*(1+scale)+shift`` -> x dtype."""
    var = torch.mean(x.float() ** 2, dim=-1, keepdim=True)
    n = x.float() * torch.rsqrt(var + eps)
    scale, shift, gate = torch.chunk(mod.float(), 3, dim=-1)
    n = n * (1 + scale) + shift
    return _r(n, policy), _r(gate, policy)


def rms_norm(x: Tensor, weight: Tensor, eps: float, policy: str) -> Tensor:
    """Plain Gemma RMSNorm (``modeling_gemma.py:94-99``): ``n * (1 + w)`` in fp32."""
    var = torch.mean(x.float() ** 2, dim=-1, keepdim=True)
    n = x.float() * torch.rsqrt(var + eps)
    return _r(n * (1.0 + weight.float()), policy)


def rope_cos_sin(position_ids: Tensor, head_dim: int, base: float, policy: str) -> Tuple[Tensor, Tensor]:
    """``GemmaRotaryEmbedding`` (``modeling_gemma.py:151-182``): fp32, cast to the hidden dtype."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    freqs = position_ids.float()[:, None] * inv_freq[None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    return _r(emb.cos(), policy), _r(emb.sin(), policy)


def apply_rope(x: Tensor, cos: Tensor, sin: Tensor, policy: str) -> Tensor:
    """RoPE on ``[T, H, D]`` with ``[T, D]`` tables, fp32 math and one rounding.

    Matches the fused epilogue of ``_qkv_rope_kernel`` (``rlinf_fused_denoise.py:262-270``):
    ``o_lo = x_lo*c - x_hi*s``, ``o_hi = x_hi*c + x_lo*s``.
    """
    half = x.shape[-1] // 2
    lo, hi = x[..., :half], x[..., half:]
    c = cos[:, None, :]
    s = sin[:, None, :]
    o_lo = lo * c[..., :half] - hi * s[..., :half]
    o_hi = hi * c[..., half:] + lo * s[..., half:]
    return _r(torch.cat([o_lo, o_hi], dim=-1), policy)


def attention(q: Tensor, k: Tensor, v: Tensor, mask_add: Tensor, scaling: float, policy: str) -> Tensor:
    """``eager_attention_forward`` (``modeling_gemma.py:252-275``) for MQA.

    q ``[T, H, D]``, k/v ``[S, D]`` (one KV head shared by all H, ``repeat_kv``),
    ``mask_add`` ``[T, S]`` additive fp32.  Scores are a bf16 GEMM output times
    ``scaling``, plus the fp32 mask, fp32 softmax, probabilities rounded to bf16,
    bf16 P@V.  Returns ``[T, H*D]``.
    """
    t, h, d = q.shape
    s = _r(torch.einsum("thd,sd->hts", q.float(), k.float()), policy) * scaling
    s = s + mask_add[None]
    p = torch.softmax(s.float(), dim=-1)
    p = _r(p, policy)
    o = _r(torch.einsum("hts,sd->thd", p, v.float()), policy)
    return o.reshape(t, h * d)


def suffix_mask(prefix_pad: Tensor, suffix_len: int) -> Tensor:
    """Denoise attention mask ``[M, P+M]`` additive (``engine.py:453-491``).

    Suffix tokens see every valid prefix token and, with ``att_masks=[1,0,...,0]``
    (``pi0_pytorch.py:344``), every suffix token.
    """
    p = prefix_pad.shape[-1]
    allow = torch.cat([prefix_pad.bool()[None, :].expand(suffix_len, p), torch.ones(suffix_len, suffix_len, dtype=torch.bool)], dim=1)
    return torch.where(allow, 0.0, MASK_NEG).float()


def prefix_mask(prefix_pad: Tensor) -> Tensor:
    """Prefix-LM mask ``[P, P]`` (all ``att_masks`` zero, ``pi0_pytorch.py:246-251,56-85``)."""
    pad = prefix_pad.bool()
    allow = pad[None, :] & pad[:, None]
    return torch.where(allow, 0.0, MASK_NEG).float()


# ---------------------------------------------------------------------------
# action expert
# ---------------------------------------------------------------------------


def expert_forward(
    w: Dict[str, Tensor],
    h: Tensor,
    kv_prefix: Sequence[Tuple[Tensor, Tensor]],
    mods: Tensor,
    position_ids: Tensor,
    mask_add: Tensor,
    depth: int,
    policy: str,
    eps: float = 1e-6,
    rope_base: float = 10000.0,
    prefix: str = "paligemma_with_expert.gemma_expert.model.",
    collect: Optional[list] = None,
) -> Tensor:
    """``GemmaModel.forward`` of the expert (``modeling_gemma.py:662-794``).

    h ``[M, width]`` (already the expert input, cast to the layer dtype), kv_prefix
    ``[depth]`` of ``(K [P, D], V [P, D])``, mods ``[n_norm, 3*width]``.  No sqrt(width)
    normaliser (``modeling_gemma.py:739-740``).  Returns the final adaRMS output
    ``[M, width]``.
    """
    h = _r(h, policy)
    nq = w[f"{prefix}layers.0.self_attn.q_proj.weight"].shape[0]
    hd = w[f"{prefix}layers.0.self_attn.k_proj.weight"].shape[0]  # one KV head
    n_heads = nq // hd
    cos, sin = rope_cos_sin(position_ids, hd, rope_base, policy)
    for i in range(depth):
        p = f"{prefix}layers.{i}."
        resid = h
        xn, gate = ada_rms_norm(h, mods[2 * i], eps, policy)
        q = _mm(xn, w[p + "self_attn.q_proj.weight"], policy).view(-1, n_heads, hd)
        k = _mm(xn, w[p + "self_attn.k_proj.weight"], policy).view(-1, 1, hd)
        v = _mm(xn, w[p + "self_attn.v_proj.weight"], policy)
        q = apply_rope(q, cos, sin, policy)
        k = apply_rope(k, cos, sin, policy).view(-1, hd)
        kk = torch.cat([kv_prefix[i][0].float(), k], dim=0)
        vv = torch.cat([kv_prefix[i][1].float(), v], dim=0)
        a = attention(q, kk, vv, mask_add, hd ** -0.5, policy)
        o = _mm(a, w[p + "self_attn.o_proj.weight"], policy)
        h = _r(resid + o * gate, policy)
        resid = h
        hn, gate2 = ada_rms_norm(h, mods[2 * i + 1], eps, policy)
        g = _mm(hn, w[p + "mlp.gate_proj.weight"], policy)
        u = hn.float() @ _r(w[p + "mlp.up_proj.weight"].float(), policy).t()
        act = _r(gelu_tanh(g) * u, policy)
        dn = _mm(act, w[p + "mlp.down_proj.weight"], policy)
        h = _r(resid + dn * gate2, policy)
        if collect is not None:
            collect.append(h.clone())
    out, _ = ada_rms_norm(h, mods[2 * depth], eps, policy)
    return out


def velocity(
    w: Dict[str, Tensor],
    x_t: Tensor,
    kv_prefix: Sequence[Tuple[Tensor, Tensor]],
    mods: Tensor,
    prefix_pad: Tensor,
    depth: int,
    policy: str,
    collect: Optional[list] = None,
) -> Tensor:
    """``get_velocity`` (``engine.py:681-768``) for one observation.

    x_t ``[M, 32]`` fp32 -> v_t ``[M, 32]`` fp32: ``action_in_proj`` (fp32), expert,
    last M rows to fp32, ``action_out_proj`` (fp32).
    """
    m = x_t.shape[0]
    emb = x_t.float() @ w["action_in_proj.weight"].t() + w["action_in_proj.bias"]
    n_valid = int(prefix_pad.sum())
    pos = torch.arange(m) + n_valid  # prefix_offsets + cumsum(ones) - 1
    mask = suffix_mask(prefix_pad, m)
    out = expert_forward(w, emb, kv_prefix, mods, pos, mask, depth, policy, collect=collect)
    return out.float() @ w["action_out_proj.weight"].t() + w["action_out_proj.bias"]


def euler(x_t: Tensor, v_t: Tensor, t: float, delta: float) -> Tensor:
    """flow_ode mean (``engine.py:664-675``), written as the reference writes it."""
    t = torch.tensor(t, dtype=torch.float32)
    delta = torch.tensor(delta, dtype=torch.float32)
    x0 = x_t - v_t * t
    x1 = x_t + v_t * (1 - t)
    return x0 * (1 - (t - delta)) + x1 * (t - delta)


def sampler_step(x_t: Tensor, v_t: Tensor, idx: int, num_steps: int, method: str, noise_level: float,
                 step_noise: Optional[Tensor]) -> Tensor:
    """``x_t_mean + noise * x_t_std`` of ``sample_mean_var_val`` for flow_sde / flow_cps
    (``_extract_src/openpi_action_model.py:984-1006``), fp32."""
    ts = timesteps(num_steps)
    t = ts[idx]
    delta = ts[idx] - ts[idx + 1]
    nl = torch.tensor(noise_level, dtype=torch.float32)
    x0 = x_t - v_t * t
    x1 = x_t + v_t * (1 - t)
    if method == "flow_sde":
        denom = torch.where(ts == 1, ts[1], ts)
        sigma = (nl * torch.sqrt(ts / (1 - denom))[:-1])[idx]
        w0 = 1 - (t - delta)
        w1 = t - delta - sigma ** 2 * delta / (2 * t)
        std = torch.sqrt(delta) * sigma
    elif method == "flow_cps":
        w0 = 1 - (t - delta)
        w1 = (t - delta) * torch.cos(torch.pi * nl / 2)
        std = (t - delta) * torch.sin(torch.pi * nl / 2)
    else:
        raise ValueError(method)
    return x0 * w0 + x1 * w1 + step_noise * std


def denoise_loop(
    w: Dict[str, Tensor],
    noise: Tensor,
    kv_prefix: Sequence[Tuple[Tensor, Tensor]],
    prefix_pad: Tensor,
    depth: int,
    num_steps: int,
    policy: str,
    table: Optional[Tensor] = None,
    prefix: str = "paligemma_with_expert.gemma_expert.model.",
    velocities: Optional[list] = None,
    method: str = "flow_ode",
    noise_level: float = 0.0,
    step_noise: Optional[Tensor] = None,
) -> Tensor:
    """The ``num_steps`` Euler loop of ``sample_actions`` (``engine.py:390-405``); a
    stochastic ``method`` adds ``step_noise[s]`` per step (``sampler_step``)."""
    if table is None:
        table = adarms_table(w, depth, num_steps, prefix)
    ts = timesteps(num_steps)
    x = noise.float()
    for s in range(num_steps):
        v = velocity(w, x, kv_prefix, table[s], prefix_pad, depth, policy)
        if velocities is not None:
            velocities.append(v.clone())
        if method == "flow_ode":
            x = euler(x, v, float(ts[s]), float(ts[s] - ts[s + 1]))
        else:
            x = sampler_step(x, v, s, num_steps, method, noise_level, step_noise[s])
    return x


# ---------------------------------------------------------------------------
# PaliGemma prefix LM (Gemma-2B, no adaRMS, KV-cache fill)
# ---------------------------------------------------------------------------


def prefix_lm_kv(
    w: Dict[str, Tensor],
    embs: Tensor,
    prefix_pad: Tensor,
    depth: int,
    policy: str,
    eps: float = 1e-6,
    rope_base: float = 10000.0,
    prefix: str = "paligemma_with_expert.paligemma.model.language_model.",
) -> List[Tuple[Tensor, Tensor]]:
    """Prefix forward with ``use_cache=True`` (``gemma_pytorch.py:131-142``).

    Same layer math as the expert with plain RMSNorm ``(1+w)`` and ungated
    residuals; q|k|v fused (``prefix_qkv_fused.py:132-139``); the last layer only
    produces K/V (``prefix_last_layer.py:46-112``).  Returns ``[depth]`` of
    ``(K [P, D], V [P, D])`` with RoPE applied to K.
    """
    h = _r(embs, policy)
    nq = w[f"{prefix}layers.0.self_attn.q_proj.weight"].shape[0]
    hd = w[f"{prefix}layers.0.self_attn.k_proj.weight"].shape[0]
    n_heads = nq // hd
    pos = torch.cumsum(prefix_pad.long(), dim=-1) - 1
    cos, sin = rope_cos_sin(pos, hd, rope_base, policy)
    mask = prefix_mask(prefix_pad)
    kv = []
    for i in range(depth):
        p = f"{prefix}layers.{i}."
        xn = rms_norm(h, w[p + "input_layernorm.weight"], eps, policy)
        k = _mm(xn, w[p + "self_attn.k_proj.weight"], policy).view(-1, 1, hd)
        v = _mm(xn, w[p + "self_attn.v_proj.weight"], policy)
        k = apply_rope(k, cos, sin, policy).view(-1, hd)
        kv.append((k, v))
        if i == depth - 1:
            break
        q = _mm(xn, w[p + "self_attn.q_proj.weight"], policy).view(-1, n_heads, hd)
        q = apply_rope(q, cos, sin, policy)
        a = attention(q, k, v, mask, hd ** -0.5, policy)
        h = _r(h + _mm(a, w[p + "self_attn.o_proj.weight"], policy), policy)
        hn = rms_norm(h, w[p + "post_attention_layernorm.weight"], eps, policy)
        g = _mm(hn, w[p + "mlp.gate_proj.weight"], policy)
        u = hn.float() @ _r(w[p + "mlp.up_proj.weight"].float(), policy).t()
        act = _r(gelu_tanh(g) * u, policy)
        h = _r(h + _mm(act, w[p + "mlp.down_proj.weight"], policy), policy)
    return kv


# ---------------------------------------------------------------------------
# SigLIP So400m/14 + projector, language embedding, prefix assembly
# ---------------------------------------------------------------------------


def layer_norm(x: Tensor, w: Tensor, b: Tensor, eps: float, policy: str) -> Tensor:
    """LayerNorm with fp32 statistics; bf16 parameters under the bf16 policy."""
    y = torch.nn.functional.layer_norm(x.float(), (x.shape[-1],), _r(w.float(), policy), _r(b.float(), policy), eps)
    return _r(y, policy)


def siglip_image_features(
    w: Dict[str, Tensor],
    images: Tensor,
    depth: int,
    policy: str,
    num_heads: int = 16,
    patch: int = 14,
    eps: float = 1e-6,
    prefix: str = "paligemma_with_expert.paligemma.model.vision_tower.vision_model.",
    proj_prefix: str = "paligemma_with_expert.paligemma.model.multi_modal_projector.linear.",
) -> Tensor:
    """SigLIP vision tower + PaliGemma projector: ``[V,3,H,W]`` -> ``[V, patches, proj]``.

    Patch conv and position embedding in fp32 (kept fp32 by
    ``gemma_pytorch.py:93-96``), 27 pre-LN encoder layers (bf16 GEMMs, fp32 LayerNorm
    and softmax), post-LN, linear projector.  Image features are NOT divided by
    sqrt(text width): pi0.5's ``embed_image`` follows the JAX model, which projects
    SigLIP's output with a plain linear head.
    """
    v_, c, hh, ww = images.shape
    gh, gw = hh // patch, ww // patch
    pw = w[prefix + "embeddings.patch_embedding.weight"]
    width = pw.shape[0]
    # im2col: [V, gh*gw, 3*patch*patch] with (c, ky, kx) order == conv weight order
    cols = images.float().reshape(v_, c, gh, patch, gw, patch).permute(0, 2, 4, 1, 3, 5).reshape(v_, gh * gw, c * patch * patch)
    x = cols @ pw.reshape(width, -1).t() + w[prefix + "embeddings.patch_embedding.bias"]
    x = x + w[prefix + "embeddings.position_embedding.weight"][None]
    h = _r(x, policy)
    hd = width // num_heads
    for i in range(depth):
        p = f"{prefix}encoder.layers.{i}."
        xn = layer_norm(h, w[p + "layer_norm1.weight"], w[p + "layer_norm1.bias"], eps, policy)
        def lin(name, a):
            wt = _r(w[p + name + ".weight"].float(), policy)
            return _r(a.float() @ wt.t() + _r(w[p + name + ".bias"].float(), policy), policy)
        q = lin("self_attn.q_proj", xn).view(v_, -1, num_heads, hd)
        k = lin("self_attn.k_proj", xn).view(v_, -1, num_heads, hd)
        vv = lin("self_attn.v_proj", xn).view(v_, -1, num_heads, hd)
        s = _r(_r(torch.einsum("bqhd,bkhd->bhqk", q, k), policy) * hd ** -0.5, policy)
        pr = _r(torch.softmax(s.float(), dim=-1), policy)
        a = _r(torch.einsum("bhqk,bkhd->bqhd", pr, vv), policy).reshape(v_, -1, width)
        h = _r(h + lin("self_attn.out_proj", a), policy)
        xn = layer_norm(h, w[p + "layer_norm2.weight"], w[p + "layer_norm2.bias"], eps, policy)
        f = _r(gelu_tanh(lin("mlp.fc1", xn)), policy)
        h = _r(h + lin("mlp.fc2", f), policy)
    h = layer_norm(h, w[prefix + "post_layernorm.weight"], w[prefix + "post_layernorm.bias"], eps, policy)
    wp = _r(w[proj_prefix + "weight"].float(), policy)
    return _r(h.float() @ wp.t() + _r(w[proj_prefix + "bias"].float(), policy), policy)


def embed_language(embed_table: Tensor, tokens: Tensor, policy: str) -> Tensor:
    """``embed_tokens(ids) * sqrt(width)`` (``pi0_pytorch.py:225-228``)."""
    e = embed_table[tokens.long()].float()
    return _r(_r(e, policy) * math.sqrt(e.shape[-1]), policy)


def embed_prefix(image_feats: Tensor, lang_emb: Tensor) -> Tensor:
    """Concatenate ``[views*patches + tokens, width]`` (``pi0_pytorch.py:190-253``)."""
    return torch.cat([image_feats.reshape(-1, image_feats.shape[-1]), lang_emb.reshape(-1, lang_emb.shape[-1])], dim=0)


# ---------------------------------------------------------------------------
# input / output transforms around sample_actions (predict_action_batch)
# ---------------------------------------------------------------------------
# The reference runs these through openpi (third-party, not in the reference
# tree): its image preprocessing (preprocess_observation_pytorch, called at
# pi0_pytorch.py:165-174, and the ResizeImages input transform) and its
# Normalize / Unnormalize transforms built at builder.py:120-136.  openpi's
# source is absent here, so the image resize is anchored on torch's
# F.interpolate (bilinear, half-pixel centres, no antialiasing) with the
# resize-with-pad geometry (aspect ratio kept, longer side fitted, centred, black
# border); parity with openpi's own resize is unpinned.


def preprocess_images(images: Tensor, size: int = 224) -> Tensor:
    """uint8 ``[n, h, w, 3]`` (or ``[n, 3, h, w]``) -> fp32 ``[n, 3, size, size]`` in [-1, 1]."""
    x = images
    if not (x.shape[1] == 3 and x.shape[-1] != 3):
        x = x.permute(0, 3, 1, 2)
    x = x.float()
    n, _, h, w = x.shape
    ratio = max(w / size, h / size)
    rh = min(max(int(h / ratio), 1), size)
    rw = min(max(int(w / ratio), 1), size)
    if (rh, rw) != (h, w):
        x = torch.nn.functional.interpolate(x, size=(rh, rw), mode="bilinear", align_corners=False, antialias=False)
    out = torch.full((n, 3, size, size), -1.0)
    py, px = (size - rh) // 2, (size - rw) // 2
    out[:, :, py: py + rh, px: px + rw] = x / 255.0 * 2.0 - 1.0
    return out


def normalize(x: Tensor, a: Tensor, b: Tensor, use_quantiles: bool, out_dim: int) -> Tensor:
    """openpi Normalize (mean/std or q01/q99) on the first ``len(a)`` features, then
    zero-padding to ``out_dim`` (PadStatesAndActions)."""
    x = x.float().clone()
    d = min(a.numel(), x.shape[-1])
    a, b = a[:d].float(), b[:d].float()
    if use_quantiles:
        x[..., :d] = (x[..., :d] - a) / (b - a + 1e-6) * 2.0 - 1.0
    else:
        x[..., :d] = (x[..., :d] - a) / (b + 1e-6)
    pad = out_dim - x.shape[-1]
    return torch.nn.functional.pad(x, (0, pad)) if pad > 0 else x


def unnormalize(x: Tensor, a: Tensor, b: Tensor, use_quantiles: bool, out_dim: int) -> Tensor:
    """openpi Unnormalize on the first ``len(a)`` features, then the policy's output
    slice ``[..., :out_dim]`` (LiberoOutputs, TurtleOutputs at
    dataconfig/policies/turtle_policy.py:89-93)."""
    x = x.float().clone()
    d = min(a.numel(), x.shape[-1])
    a, b = a[:d].float(), b[:d].float()
    if use_quantiles:
        x[..., :d] = (x[..., :d] + 1.0) / 2.0 * (b - a + 1e-6) + a
    else:
        x[..., :d] = x[..., :d] * (b + 1e-6) + a
    return x[..., :out_dim]
