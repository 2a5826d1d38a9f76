"""``OpenPi0Inference`` (alias ``Engine``): the reference's engine API on B200 kernels.

Mirrors ``pi05_infer/engine.py`` of the reference:

* ``sample_actions(observation, noise=None) -> {"actions": [B, 50, 32] fp32}``
  (``engine.py:344-406``): prefix (SigLIP + language embedding + Gemma-2B prefix
  LM filling the static KV cache) then ``num_steps`` Euler steps of the action
  expert, all enqueued through the C ABI and replayed as CUDA graphs.
* ``predict_action_batch(env_obs)`` (``engine.py:321-342``) for dict observations.
* ``enable_torch_compile(mode)`` (``engine.py:1003``): accepted for API
  compatibility; the kernels are compiled ahead of time, so it does nothing.
* ``capture_cuda_graph(train_bs, eval_bs)`` (``engine.py:831``): enables graph
  replay (on by default).
* ``invalidate_weight_derived_caches()`` (``engine.py:526-554``): after an
  in-place weight update, re-packs every derived device buffer in place (fused
  QKV, stacked adaRMS dense, modulation table) so captured graphs stay valid.

There is no CPU or eager fallback: without the built library every call raises.
"""

from __future__ import annotations

import dataclasses
import math
from typing import Any, Dict, Optional

import torch

from . import _lib, abi, ops, synthetic, transforms
from .config import ACTION_DIM, ACTION_HORIZON, GEMMA_2B, GEMMA_300M, SIGLIP_SO400M, EngineConfig
from .expert import DenoiseRunner, ExpertWeights
from .prefix import PrefixRunner, PrefixWeights, embed_tokens
from .transforms import NormStats


@dataclasses.dataclass
class Observation:
    """openpi ``Observation`` fields used by ``sample_actions`` (openpi is not a dependency)."""

    images: Dict[str, torch.Tensor]          # name -> [B, 3, 224, 224] float in [-1, 1]
    image_masks: Dict[str, torch.Tensor]     # name -> [B] bool
    tokenized_prompt: torch.Tensor           # [B, L] int
    tokenized_prompt_mask: torch.Tensor      # [B, L] bool
    state: torch.Tensor                      # [B, 32]

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "Observation":
        return cls(images=d["image"], image_masks=d["image_mask"], tokenized_prompt=d["tokenized_prompt"],
                   tokenized_prompt_mask=d["tokenized_prompt_mask"], state=d["state"])


def _slice_observation(obs: Observation, i: int) -> Observation:
    """Observation ``i`` of a batch, with its leading batch dimension kept (size 1)."""
    sl = slice(i, i + 1)
    return Observation({k: v[sl] for k, v in obs.images.items()}, {k: v[sl] for k, v in obs.image_masks.items()},
                       obs.tokenized_prompt[sl], obs.tokenized_prompt_mask[sl],
                       obs.state[sl] if obs.state is not None else None)


class OpenPi0Inference:
    """pi0.5 inference engine on one GPU (one engine per GPU for replicas)."""

    def __init__(self, config: Optional[EngineConfig] = None, state_dict: Optional[Dict[str, torch.Tensor]] = None,
                 device="cuda", prefix_len: int = 968, num_views: int = 3, prompt_len: int = 200):
        if not torch.cuda.is_available():
            raise RuntimeError("pi05_infer needs a CUDA device (sm_100a); there is no CPU path")
        self.config = config or EngineConfig()
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        _lib.lib()
        self.num_views = num_views
        self.prompt_len = prompt_len
        self.prefix_len = prefix_len
        self.state_dict = state_dict
        self.use_cuda_graph = True
        self.expert = None
        self.prefix_w = None
        self.vision = None
        self.embed_table = None
        self._denoise = None
        self._prefix = None
        self._graphs = {}
        self._kv_host = None      # host copy of the key masks last written to the device
        self._kv_pinned = None
        self._ids_pinned = None   # pinned int32 staging of the prompt ids
        self._ids_event = None
        self._inputs_read = None  # event after the input copies of the last call
        self.norm_stats: Optional[Dict[str, NormStats]] = None
        self._batched: Dict[int, DenoiseRunner] = {}  # batch size -> batched denoise runner
        self._bstatic: Dict[int, Dict[str, torch.Tensor]] = {}  # batch size -> static inputs
        self._bsiglip: Dict[int, Any] = {}  # batch size -> SiglipRunner over all its views
        if state_dict is not None:
            self.load_state_dict(state_dict)

    # ------------------------------------------------------------------ weights
    @classmethod
    def synthetic(cls, device="cuda", seed: int = 0, with_vision: bool = False, with_prefix: bool = True,
                  config: Optional[EngineConfig] = None, num_views: int = 3, prompt_len: int = 200
                  ) -> "OpenPi0Inference":
        """Random-init weights (N(0, 0.02)) drawn on the device (benchmarks, smoke tests);
        the prefix holds ``num_views`` x 256 image tokens and ``prompt_len`` text tokens."""
        dev = torch.device(device)
        sd = {}
        sd.update(synthetic.make_expert_weights(seed, GEMMA_300M, device=dev))
        if with_prefix:
            sd.update(synthetic.make_prefix_lm_weights(seed + 10, GEMMA_2B, device=dev, with_embedding=with_vision))
        if with_vision:
            sd.update(synthetic.make_siglip_weights(seed + 20, device=dev))
        npatch = (config or EngineConfig()).siglip.num_patches
        eng = cls(config, sd, device=dev, prefix_len=num_views * npatch + prompt_len, num_views=num_views,
                  prompt_len=prompt_len)
        return eng

    def load_state_dict(self, sd: Dict[str, torch.Tensor]) -> None:
        self.state_dict = sd
        if self.expert is None:
            self.expert = ExpertWeights(sd, self.config.expert, self.device)
        else:
            self.expert.load(sd)
        lm_key = synthetic.LM_PREFIX + "layers.0.self_attn.q_proj.weight"
        if lm_key in sd:
            if self.prefix_w is None:
                self.prefix_w = PrefixWeights(sd, self.config.prefix_lm, self.device)
            else:
                self.prefix_w.load(sd)
        if synthetic.EMBED_KEY in sd:
            t = sd[synthetic.EMBED_KEY]
            if self.embed_table is None:
                self.embed_table = t.to(device=self.device, dtype=torch.bfloat16).contiguous()
            else:
                self.embed_table.copy_(t)
        vkey = synthetic.VISION_PREFIX + "embeddings.patch_embedding.weight"
        if vkey in sd:
            from .vision import SiglipWeights

            if self.vision is None:
                self.vision = SiglipWeights(sd, self.config.siglip, self.device)
            else:
                self.vision.load(sd)

    def invalidate_weight_derived_caches(self) -> None:
        """Re-pack every derived buffer from ``self.state_dict`` in place (engine.py:526-554)."""
        if self.state_dict is None:
            return
        self.load_state_dict(self.state_dict)
        for den in [self._denoise, *self._batched.values()]:
            if den is not None:
                den.build_table()

    # ------------------------------------------------------------ compat knobs
    def enable_torch_compile(self, mode: str = "max-autotune") -> None:  # noqa: ARG002
        """Kernels are compiled ahead of time; kept for API compatibility."""
        return None

    def capture_cuda_graph(self, train_bs: Optional[int] = None, eval_bs: Optional[int] = None) -> None:  # noqa: ARG002
        self.use_cuda_graph = True

    def is_cuda_graph_enabled(self) -> bool:
        return self.use_cuda_graph

    # ------------------------------------------------------------- components
    def _runners(self):
        if self._denoise is None:
            self._denoise = DenoiseRunner(self.expert, prefix_len=self.prefix_len, num_steps=self.config.num_steps,
                                          horizon=self.config.action_horizon, action_dim=self.config.action_dim,
                                          noise_method=self.config.noise_method,
                                          noise_level=self.config.noise_level)
        if self._prefix is None and self.prefix_w is not None:
            self._prefix = PrefixRunner(self.prefix_w, self.prefix_len, self._denoise.k_cache, self._denoise.v_cache)
        return self._prefix, self._denoise

    def prefill_from_embeddings(self, embs: torch.Tensor, valid: Optional[torch.Tensor] = None) -> None:
        """Run the prefix LM over given prefix embeddings ``[P, 2048]`` (config 2)."""
        prefix, den = self._runners()
        if prefix is None:
            raise RuntimeError("engine has no prefix-LM weights")
        if valid is None:
            valid = torch.ones(self.prefix_len, dtype=torch.bool, device=self.device)
        prefix.run(embs.to(self.device, torch.bfloat16), valid.to(self.device))
        den.key_valid[: self.prefix_len].copy_(valid.reshape(-1).to(torch.uint8))
        den.key_valid[self.prefix_len:].fill_(1)

    def set_prefix_kv(self, kv, valid: torch.Tensor) -> None:
        """Use a precomputed prefix cache ``[(K, V)]`` (config 1)."""
        _, den = self._runners()
        den.set_prefix(kv, valid.to(self.device))

    def _embed_prefix(self, obs: Observation) -> torch.Tensor:
        """SigLIP image tokens + scaled language embeddings -> prefix buffer (pi0_pytorch.py:190-253)."""
        prefix, den = self._runners()
        if self.vision is None or self.embed_table is None:
            raise RuntimeError("engine has no SigLIP / embedding weights")
        from .vision import SiglipRunner

        if not hasattr(self, "_siglip"):
            self._siglip = SiglipRunner(self.vision, self.num_views)
        names = list(obs.images.keys())
        imgs = torch.cat([obs.images[n].to(self.device, torch.float32) for n in names], 0)
        npatch = self.config.siglip.num_patches
        self._siglip.run(imgs, out=prefix.h[: len(names) * npatch])
        ids = obs.tokenized_prompt.reshape(-1).to(self.device, torch.int32)
        if not hasattr(self, "_ids"):
            self._ids = torch.zeros(self.prompt_len, dtype=torch.int32, device=self.device)
        self._ids.copy_(ids)
        base = len(names) * npatch
        embed_tokens(self.embed_table, self._ids, prefix.h[base: base + self.prompt_len],
                     math.sqrt(self.embed_table.shape[1]), ops.workspace(self.device), abi.stream_of(self.device))
        return self._prefix_valid(obs)

    def _prefix_valid(self, obs: Observation) -> torch.Tensor:
        """Key-validity of the prefix: every patch of a present view, then the prompt mask."""
        npatch = self.config.siglip.num_patches
        return torch.cat([obs.image_masks[n].to(self.device).reshape(-1, 1).expand(-1, npatch).reshape(-1)
                          for n in obs.images] + [obs.tokenized_prompt_mask.reshape(-1).to(self.device)])

    def _host_key_valid(self, obs: Observation) -> Optional[torch.Tensor]:
        """The prefix key-validity mask built on the host (uint8), or None when a mask
        of the observation lives on the device."""
        npatch = self.config.siglip.num_patches
        parts = []
        for n in obs.images:
            m = obs.image_masks[n]
            if m.is_cuda:
                return None
            parts.append(m.reshape(-1, 1).expand(-1, npatch).reshape(-1))
        pm = obs.tokenized_prompt_mask
        if pm.is_cuda:
            return None
        parts.append(pm.reshape(-1))
        return torch.cat(parts).to(torch.uint8)

    def _refresh_key_valid(self, obs: Observation) -> None:
        """Key masks of the captured pipeline: built on the host and copied (pinned,
        asynchronously) only when they differ from the last call's."""
        hv = self._host_key_valid(obs)
        if hv is None:
            self._set_key_valid(self._prefix_valid(obs))
            return
        if self._kv_host is not None and torch.equal(hv, self._kv_host):
            return
        prefix, den = self._runners()
        pinned = hv.pin_memory()
        prefix.key_valid.copy_(pinned, non_blocking=True)
        den.key_valid[: self.prefix_len].copy_(pinned, non_blocking=True)
        self._kv_host, self._kv_pinned = hv, pinned  # the pinned copy stays alive until replaced

    def _set_key_valid(self, valid: torch.Tensor) -> None:
        self._kv_host = None  # the device masks no longer match the host cache
        prefix, den = self._runners()
        prefix.key_valid.copy_(valid.to(torch.uint8))
        den.key_valid[: self.prefix_len].copy_(valid.to(torch.uint8))
        den.key_valid[self.prefix_len:].fill_(1)

    # ------------------------------------------------------------ public API
    @torch.no_grad()
    def sample_actions(self, observation: Observation, noise: Optional[torch.Tensor] = None) -> dict:
        """Full inference: prefix cache + ``num_steps`` flow_ode Euler steps (engine.py:344-406).

        ``bsize = observation.state.shape[0]`` (``engine.py:350``); ``noise`` is
        ``[bsize, action_horizon, action_dim]`` or None (drawn N(0, 1) on the device).
        Observations of a batch are independent: each runs the captured pipeline
        in turn on this engine's GPU.  Returns ``{"actions": [bsize, H, 32]}`` fp32 on
        the device.  The caller's (pinned) input buffers have been read when this
        returns, so they may be reused at once."""
        bsize = int(observation.state.shape[0]) if observation.state is not None and observation.state.dim() > 1 \
            else int(observation.tokenized_prompt.shape[0])
        h, a = self.config.action_horizon, self.config.action_dim
        if noise is None:
            noise = torch.randn((bsize, h, a), dtype=torch.float32, device=self.device)
        noise = noise.reshape(-1, h, a)
        if noise.shape[0] != bsize:
            raise ValueError(f"noise has batch {noise.shape[0]}, observation has {bsize}")
        if bsize == 1:
            return {"actions": self._sample_one(observation, noise[0])}
        if self.vision is not None and self.embed_table is not None:
            return {"actions": self._sample_batched(observation, noise)}
        outs = [self._sample_one(_slice_observation(observation, i), noise[i]) for i in range(bsize)]
        return {"actions": torch.cat(outs, 0)}

    # -------------------------------------------------------- batched observations
    def _batched_runner(self, bsize: int) -> DenoiseRunner:
        r = self._batched.get(bsize)
        if r is None:
            _, den1 = self._runners()
            r = DenoiseRunner(self.expert, prefix_len=self.prefix_len, num_steps=self.config.num_steps,
                              horizon=self.config.action_horizon, action_dim=self.config.action_dim, batch=bsize,
                              fold_source=den1, noise_method=self.config.noise_method,
                              noise_level=self.config.noise_level)
            self._batched[bsize] = r
        return r

    def _host_batch_key_valid(self, obs: Observation, bsize: int, kv_rows: int) -> torch.Tensor:
        """Key masks of a batch, uint8 ``[bsize, kv_rows]``: the views' patches, the
        prompt mask, then the action tokens (always valid)."""
        npatch = self.config.siglip.num_patches
        parts = [obs.image_masks[n].reshape(bsize, 1).cpu().expand(bsize, npatch) for n in obs.images]
        parts.append(obs.tokenized_prompt_mask.reshape(bsize, -1).cpu())
        parts.append(torch.ones(bsize, kv_rows - self.prefix_len, dtype=torch.bool))
        return torch.cat(parts, 1).to(torch.uint8)

    def _enqueue_batched(self, den: DenoiseRunner, bsize: int, stream: int) -> None:
        """SigLIP over every view of the batch in one pass, then the embeddings and the
        prefix LM of each observation into its own cache (the prefix runner
        re-targeted at observation b's cache views), then one batched Euler loop over
        all of them."""
        prefix, den1 = self._runners()
        npatch = self.config.siglip.num_patches
        nv = self.num_views
        st = self._bstatic[bsize]
        base = nv * npatch
        depth = self.config.expert.depth
        self._bsiglip[bsize].enqueue(st["imgs"], st["feats"], stream)
        for b in range(bsize):
            prefix.h[:base].copy_(st["feats"][b * base: (b + 1) * base])
            embed_tokens(self.embed_table, st["ids"][b], prefix.h[base: base + self.prompt_len],
                         math.sqrt(self.embed_table.shape[1]), ops.workspace(self.device), stream)
            caches = [den.cache(i, b) for i in range(depth)]
            prefix.target([c[0] for c in caches], [c[1] for c in caches], den.key_valid_of(b))
            prefix.enqueue(stream)
        prefix.target(den1.k_cache, den1.v_cache)
        den._enqueue(stream)

    def _sample_batched(self, observation: Observation, noise: torch.Tensor) -> torch.Tensor:
        """``bsize`` observations through one batched pipeline: the denoise GEMMs run at
        bsize x 50 token rows, so the expert weights stream once per step for the batch."""
        from .vision import SiglipRunner

        bsize = noise.shape[0]
        self._runners()
        den = self._batched_runner(bsize)
        names = list(observation.images.keys())
        if len(names) != self.num_views:
            raise ValueError(f"expected {self.num_views} camera views, got {len(names)}")
        st = self._bstatic.get(bsize)
        if st is None:
            nrows = bsize * self.num_views * self.config.siglip.num_patches
            # the tower over all bsize x views images at once (its GEMMs then fill the
            # GPU); the batch's images are written straight into its input buffer
            self._bsiglip[bsize] = SiglipRunner(self.vision, bsize * self.num_views)
            st = {"imgs": self._bsiglip[bsize].images,
                  "ids": torch.zeros((bsize, self.prompt_len), dtype=torch.int32, device=self.device),
                  "feats": torch.zeros((nrows, self.config.prefix_lm.width), dtype=torch.bfloat16,
                                       device=self.device)}
            self._bstatic[bsize] = st
        imgs = st["imgs"].view(bsize, self.num_views, *st["imgs"].shape[1:])
        for i, n in enumerate(names):
            imgs[:, i].copy_(observation.images[n], non_blocking=True)
        st["ids"].copy_(observation.tokenized_prompt.reshape(bsize, -1).to(torch.int32), non_blocking=True)
        den.key_valid.copy_(self._host_batch_key_valid(observation, bsize, den.kv_rows).reshape(-1),
                            non_blocking=True)
        den.x_t.copy_(noise.reshape(den.rows, den.action_dim), non_blocking=True)
        stream = torch.cuda.current_stream(self.device)
        inputs_read = torch.cuda.Event()
        inputs_read.record(stream)
        den.draw_step_noise()
        if self.use_cuda_graph:
            g = self._graphs.get(("batch", bsize))
            if g is None:
                saved = den.x_t.clone()
                self._enqueue_batched(den, bsize, stream.cuda_stream)  # warm-up outside the capture
                torch.cuda.synchronize(self.device)
                den.x_t.copy_(saved)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self._enqueue_batched(den, bsize, torch.cuda.current_stream(self.device).cuda_stream)
                self._graphs[("batch", bsize)] = g
            g.replay()
        else:
            self._enqueue_batched(den, bsize, stream.cuda_stream)
        out = den.x_t.clone().reshape(bsize, self.config.action_horizon, self.config.action_dim)
        inputs_read.synchronize()  # the caller's input buffers have been read
        return out

    def _sample_one(self, observation: Observation, noise: torch.Tensor) -> torch.Tensor:
        prefix, den = self._runners()
        for n, img in observation.images.items():
            if img.shape[0] != 1:
                raise ValueError(f"image {n!r}: expected one observation, got batch {img.shape[0]}")
        if self.use_cuda_graph and self.vision is not None and self.embed_table is not None:
            # The whole pipeline (SigLIP, embeddings, prefix LM, Euler loop) replays as
            # one CUDA graph captured on the first call; each call only refreshes its
            # static inputs (images, prompt ids, key masks, noise).
            key = (tuple(observation.images.keys()), tuple(observation.images[n].shape for n in observation.images))
            if self._graphs.get("full") is None or getattr(self, "_full_key", None) != key:
                self._set_key_valid(self._prefix_valid(observation))
                self.capture_full(observation, noise.to(self.device).float())
                self._full_key = key
            stream = torch.cuda.current_stream(self.device)
            # Images first: their copy (1.8 MB) overlaps the host work that follows.
            for i, n in enumerate(observation.images):
                self._static_imgs[i: i + 1].copy_(observation.images[n], non_blocking=True)
            self._refresh_key_valid(observation)
            ids = observation.tokenized_prompt.reshape(-1)
            if ids.is_cuda:
                self._ids.copy_(ids)
            else:
                # int32 on the host into a pinned buffer, then one asynchronous copy;
                # the buffer is rewritten only after the previous call's copy read it.
                if self._ids_pinned is None or self._ids_pinned.numel() != ids.numel():
                    self._ids_pinned = torch.empty(ids.numel(), dtype=torch.int32).pin_memory()
                    self._ids_event = torch.cuda.Event()
                else:
                    self._ids_event.synchronize()
                self._ids_pinned.copy_(ids)
                self._ids.copy_(self._ids_pinned, non_blocking=True)
                self._ids_event.record(stream)
            den.x_t.copy_(noise.reshape(den.horizon, den.action_dim), non_blocking=True)
            if self._inputs_read is None:
                self._inputs_read = torch.cuda.Event()
            self._inputs_read.record(stream)
            den.draw_step_noise()  # stochastic samplers: fresh per-step noise
            self._graphs["full"].replay()
            actions = den.x_t.clone()
            # The caller's buffers were copied by the work before the replay; wait for
            # those copies only (the graph keeps running).
            self._inputs_read.synchronize()
        else:
            valid = self._embed_prefix(observation)
            self._set_key_valid(valid)
            prefix.enqueue(abi.stream_of(self.device))
            actions = den.run(noise.to(self.device, non_blocking=True).float(), use_graph=self.use_cuda_graph).clone()
            torch.cuda.current_stream(self.device).synchronize()
        return actions.reshape(1, self.config.action_horizon, self.config.action_dim)

    @torch.no_grad()
    def denoise(self, noise: Optional[torch.Tensor] = None) -> dict:
        """The Euler loop over the current prefix cache (config 2): noise -> actions."""
        _, den = self._runners()
        if noise is None:
            noise = torch.randn((self.config.action_horizon, self.config.action_dim), device=self.device)
        actions = den.run(noise.to(self.device, non_blocking=True).float(), use_graph=self.use_cuda_graph)
        return {"actions": actions.clone().reshape(1, self.config.action_horizon, self.config.action_dim)}

    # ---------------------------------------------------- input / output transforms
    def set_norm_stats(self, stats: Optional[Dict[str, "NormStats"]], use_quantiles: Optional[bool] = None) -> None:
        """Statistics for the state normalisation and the action un-normalisation
        (``norm_stats.json`` of the checkpoint, ``builder.py:112-136``)."""
        self.norm_stats = stats
        if use_quantiles is not None:
            self.config.use_quantile_norm = use_quantiles

    def obs_processor(self, env_obs: Dict[str, Any]) -> Observation:
        """Environment observation -> model observation, on the GPU (``engine.py:287-303``
        and the policy's input transform): ``main_images`` / ``wrist_images`` /
        ``extra_view_images`` uint8 ``[B, H, W, 3]`` (extra views ``[B, n, H, W, 3]``) map
        to the three camera slots and are resized / scaled to [-1, 1]
        (``pi05_preprocess_images``); ``states`` ``[B, s]`` are normalised and padded
        to the action dimension.  Prompt tokenisation stays with the caller:
        ``tokenized_prompt`` / ``tokenized_prompt_mask`` ``[B, L]``."""
        size = self.config.siglip.image_size

        def prep(x):
            x = torch.as_tensor(x)
            return transforms.preprocess_images(x.to(self.device, non_blocking=True), size)

        main = prep(env_obs["main_images"])
        b = main.shape[0]
        slots = [main]
        wrist = env_obs.get("wrist_images")
        extra = env_obs.get("extra_view_images")
        if self.config.policy == "turtle":
            views = []
            if extra is not None:
                extra = torch.as_tensor(extra)
                views = [prep(extra[:, i]) for i in range(extra.shape[1])] if extra.dim() == 5 else [prep(extra)]
            slots += views[:2]
        else:
            if wrist is not None:
                slots.append(prep(wrist))
            if extra is not None:
                slots.append(prep(extra))
        names = ["base_0_rgb", "left_wrist_0_rgb", "right_wrist_0_rgb"][: self.num_views]
        images, masks = {}, {}
        for i, n in enumerate(names):
            present = i < len(slots)
            images[n] = slots[i] if present else torch.full_like(main, -1.0)  # zero image = -1 after scaling
            masks[n] = torch.full((b,), present, dtype=torch.bool)
        stats = getattr(self, "norm_stats", None)
        st = transforms.normalize_state(torch.as_tensor(env_obs["states"]).to(self.device),
                                        None if stats is None else stats.get("state"),
                                        self.config.use_quantile_norm, self.config.action_dim)
        return Observation(images, masks, torch.as_tensor(env_obs["tokenized_prompt"]),
                           torch.as_tensor(env_obs["tokenized_prompt_mask"]).bool(), st)

    def output_transform(self, actions: torch.Tensor) -> torch.Tensor:
        """Model actions ``[B, H, 32]`` -> environment actions ``[B, action_chunk,
        env_action_dim]``: un-normalised with the action statistics and cut to the
        robot's action dimension (``engine.py:270-284``, ``LiberoOutputs`` /
        ``TurtleOutputs``)."""
        stats = getattr(self, "norm_stats", None)
        out = transforms.unnormalize_actions(actions, None if stats is None else stats.get("actions"),
                                             self.config.use_quantile_norm, self.config.env_action_dim)
        return out[:, : self.config.action_chunk]

    def predict_action_batch(self, env_obs: Dict[str, Any]) -> torch.Tensor:
        """Environment observations -> environment actions (``engine.py:321-342``):
        ``obs_processor`` (GPU preprocessing), ``sample_actions``, ``output_transform``.
        A dict that already holds openpi ``Observation`` keys (``image``,
        ``image_mask``, ``state``, ...) skips the input transform."""
        if "image" in env_obs:
            obs = Observation.from_dict(env_obs)
        else:
            obs = self.obs_processor(env_obs)
        return self.output_transform(self.sample_actions(obs)["actions"])

    # ------------------------------------------------------------ bench hooks
    def synthetic_observation(self, seed: int = 100) -> Observation:
        """Seeded synthetic observation in pinned host memory (the form a serving
        client hands over; pinned images copy to the device asynchronously)."""
        g = torch.Generator().manual_seed(seed)
        imgs = {f"cam{i}": (torch.rand((1, 3, 224, 224), generator=g) * 2 - 1).pin_memory()
                for i in range(self.num_views)}
        masks = {k: torch.ones(1, dtype=torch.bool) for k in imgs}
        toks = torch.randint(0, synthetic.VOCAB_SIZE, (1, self.prompt_len), generator=g)
        return Observation(imgs, masks, toks, torch.ones(1, self.prompt_len, dtype=torch.bool),
                           torch.randn(1, ACTION_DIM, generator=g))

    def observation_host_bytes(self, obs: Observation) -> int:
        n = sum(t.numel() * t.element_size() for t in obs.images.values())
        n += obs.tokenized_prompt.numel() * 4 + obs.tokenized_prompt_mask.numel()
        return n

    def prepare(self, obs: Observation, embed_seed: int = 3) -> None:
        """Fill the prefix cache once: from SigLIP + tokens when vision weights are
        loaded (config 3), else from N(0,1) prefix embeddings (config 2)."""
        prefix, den = self._runners()
        if self.vision is not None and self.embed_table is not None:
            valid = self._embed_prefix(obs)
            prefix.key_valid.copy_(valid.to(torch.uint8))
            prefix.enqueue(abi.stream_of(self.device))
            den.key_valid[: self.prefix_len].copy_(valid.to(torch.uint8))
        else:
            g = torch.Generator(device=self.device).manual_seed(embed_seed)
            embs = torch.randn((self.prefix_len, self.config.prefix_lm.width), generator=g, device=self.device)
            self.prefill_from_embeddings(embs)
        torch.cuda.synchronize(self.device)

    def capture_denoise(self, noise: torch.Tensor):
        """Capture the Euler loop as one CUDA graph; returns a zero-arg replay callable."""
        _, den = self._runners()
        den.x_t.copy_(noise.reshape(den.horizon, den.action_dim))
        den.capture()
        g = den.graph

        def step():
            den.x_t.copy_(noise.reshape(den.horizon, den.action_dim))
            g.replay()

        return step

    def capture_full(self, obs: Observation, noise: torch.Tensor):
        """Capture prefix + loop (device-resident inputs) as one CUDA graph."""
        prefix, den = self._runners()
        self._embed_prefix(obs)
        stream = torch.cuda.Stream(self.device)
        imgs = torch.cat([obs.images[n].to(self.device, torch.float32) for n in obs.images], 0)
        self._static_imgs = imgs
        den.x_t.copy_(noise.reshape(den.horizon, den.action_dim))

        def enqueue(st):
            self._siglip.enqueue(self._static_imgs, prefix.h, st)
            embed_tokens(self.embed_table, self._ids, prefix.h[self.num_views * 256: self.num_views * 256 + self.prompt_len],
                         math.sqrt(self.embed_table.shape[1]), ops.workspace(self.device), st)
            prefix.enqueue(st)
            den._enqueue(st)

        enqueue(abi.stream_of(self.device))
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            enqueue(torch.cuda.current_stream(self.device).cuda_stream)
        self._graphs["full"] = g
        self._full_key = (tuple(obs.images.keys()), tuple(obs.images[n].shape for n in obs.images))

        def step():
            den.x_t.copy_(noise.reshape(den.horizon, den.action_dim))
            g.replay()

        return step

    def capture_stage(self, stage: str):
        """Capture one stage of the captured pipeline alone as a CUDA graph (after
        ``capture_full``): "siglip" (the views -> image tokens of the prefix) or
        "prefix" (the prefix LM over the current prefix embeddings, which are
        restored before every replay).  Returns a zero-arg replay callable."""
        prefix, den = self._runners()
        st = torch.cuda.current_stream(self.device)
        if stage == "siglip":
            def enqueue(s):
                self._siglip.enqueue(self._static_imgs, prefix.h, s)
        elif stage == "prefix":
            saved = prefix.h.clone()

            def enqueue(s):
                prefix.h.copy_(saved)
                prefix.enqueue(s)
        else:
            raise ValueError(stage)
        enqueue(st.cuda_stream)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            enqueue(torch.cuda.current_stream(self.device).cuda_stream)
        self._graphs[stage] = g
        return g.replay

    def _time_per_layer(self, launch, reps: int) -> float:
        """Mean µs of ``launch(layer)`` over all expert layers, captured once in a
        CUDA graph and replayed ``reps`` times (CUDA events on the replay stream)."""
        st = torch.cuda.current_stream(self.device)
        for L in self.expert.layers:
            launch(L)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for L in self.expert.layers:
                launch(L)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize(self.device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            g.replay()
        e1.record(st)
        torch.cuda.synchronize(self.device)
        del g
        return e0.elapsed_time(e1) * 1e3 / (reps * len(self.expert.layers))

    def time_geglu_kernel(self, reps: int = 20) -> dict:
        """The gate/up+GeGLU GEMM alone: one launch per expert layer (302 MB of
        weights > L2)."""
        _, den = self._runners()
        s = self.expert.shape
        us = self._time_per_layer(lambda L: ops.geglu(den.xn, L["w_gate"], L["w_up"], out=den.act), reps)
        m = self.config.action_horizon
        nbytes = 2 * s.mlp_dim * s.width * 2 + m * s.width * 2 + m * s.mlp_dim * 2
        return {"us": us, "bytes": nbytes, "launches": reps * len(self.expert.layers)}

    def time_down_kernel(self, reps: int = 20) -> dict:
        """The down projection + gated residual GEMM alone: one launch per expert
        layer (151 MB of weights > L2 between replays of the same layer)."""
        _, den = self._runners()
        s = self.expert.shape
        gate = torch.ones(s.width, dtype=torch.float32, device=self.device)
        us = self._time_per_layer(
            lambda L: ops.linear_gated_residual(den.act, L["w_down"], den.h, gate, out=den.h), reps)
        m = self.config.action_horizon
        nbytes = s.width * s.mlp_dim * 2 + m * s.mlp_dim * 2 + 2 * m * s.width * 2 + s.width * 4
        return {"us": us, "bytes": nbytes, "launches": reps * len(self.expert.layers)}

    def denoise_step_bytes(self) -> int:
        """Algorithmic HBM bytes of one Euler step: expert weights + KV read + KV tail
        write + the step's adaRMS rows + action in/out projections."""
        s = self.expert.shape
        kv_len = self.prefix_len + self.config.action_horizon
        w = self.expert.nbytes_streamed_per_step()
        kv_read = s.depth * 2 * kv_len * s.head_dim * 2
        kv_write = s.depth * 2 * self.config.action_horizon * s.head_dim * 2
        mods = self.expert.n_norm * 3 * s.width * 4
        io = 2 * s.width * ACTION_DIM * 4
        return w + kv_read + kv_write + mods + io

    def last_denoise_step_us(self, loop_ms: Optional[float]) -> Optional[float]:
        if loop_ms is None:
            return None
        return loop_ms * 1e3 / self.config.num_steps

    def release_graphs(self) -> None:
        self._graphs.clear()
        for den in self._batched.values():
            den.graph = None
        if self._denoise is not None:
            self._denoise.graph = None


Engine = OpenPi0Inference
EngineConfig = EngineConfig
