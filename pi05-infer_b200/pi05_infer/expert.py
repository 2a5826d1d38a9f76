"""Action-expert denoise loop on the C ABI: weights, static buffers, graph capture.

Device layout (all allocated once by torch, never by the library):

* GEMM weights bf16 in the reference layout: ``w_qkv`` = cat(q, k, v) rows
  ``[2560, 1024]`` (``modeling_gemma.py:331-351``), ``w_o [1024, 2048]``,
  ``w_gate``/``w_up [4096, 1024]``, ``w_down [1024, 4096]`` per layer.
* fp32 (the reference keeps them fp32, ``gemma_pytorch.py:93-104``): action
  in/out projections, time MLP, the 37 adaRMS ``dense`` layers stacked in forward
  order ``[37*3072, 1024]`` (``modeling_gemma.py:577-603``) and the per-step
  modulation table ``[num_steps, 37, 3072]`` (``engine.py:556-599``).
* Static KV cache per layer ``[1, kv_rows, 256]`` bf16, prefix rows filled once per
  predict, suffix rows rewritten by every step (``modeling_gemma.py:312-329``).
* Activations ``h``/``xn`` ``[50, 1024]``, ``q [50, 8, 256]``, ``attn [50, 2048]``,
  ``act [50, 4096]`` bf16; ``x_t``/``v_t [50, 32]`` fp32.
"""

from __future__ import annotations

import ctypes
import math
import os
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import abi, ops
from .config import GemmaShape, GEMMA_300M
from .synthetic import EXPERT_PREFIX


def rope_inv_freq(head_dim: int, base: float, device) -> torch.Tensor:
    """inv_freq exactly as ``ROPE_INIT_FUNCTIONS['default']`` computes it (fp32)."""
    inv = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    return inv.to(device)


def timesteps(num_steps: int) -> torch.Tensor:
    """``[1, ..., 1/N, 0]`` as ``OpenPi0Inference._get_timesteps`` builds it (engine.py:411-429)."""
    ts = torch.linspace(1, 1 / num_steps, num_steps)
    return torch.cat([ts, torch.zeros(1)])


SAMPLERS = ("flow_ode", "flow_sde", "flow_cps")


def sampler_coefs(num_steps: int, method: str, noise_level: float) -> torch.Tensor:
    """Per-step sampler update ``x <- x0 * c0 + x1 * c1 + c2 * noise`` with
    ``x0 = x - v t``, ``x1 = x + v (1 - t)``: fp32 ``[num_steps, 3]``, computed as
    ``sample_mean_var_val`` computes the mean weights and the std
    (``_extract_src/openpi_action_model.py:984-1006``; the inference engine keeps only
    flow_ode, ``engine.py:629-676``)."""
    if method not in SAMPLERS:
        raise ValueError(f"noise_method {method!r} not supported ({SAMPLERS})")
    ts = timesteps(num_steps)
    t = ts[:-1]
    delta = ts[:-1] - ts[1:]
    nl = torch.tensor(noise_level, dtype=torch.float32)
    if method == "flow_ode":
        c0, c1, sd = 1 - (t - delta), t - delta, torch.zeros_like(t)
    elif method == "flow_sde":
        denom = torch.where(ts == 1, ts[1], ts)
        sigmas = nl * torch.sqrt(ts / (1 - denom))[:-1]
        c0 = torch.ones_like(t) - (t - delta)
        c1 = t - delta - sigmas ** 2 * delta / (2 * t)
        sd = torch.sqrt(delta) * sigmas
    else:  # flow_cps
        cos_term = torch.cos(torch.pi * nl / 2)
        sin_term = torch.sin(torch.pi * nl / 2)
        c0 = torch.ones_like(t) - (t - delta)
        c1 = (t - delta) * cos_term
        sd = (t - delta) * sin_term
    return torch.stack([c0, c1, sd], 1).to(torch.float32).contiguous()


class ExpertWeights:
    """Device copies of the action expert and its glue, packed for the kernels."""

    def __init__(self, sd: Dict[str, torch.Tensor], shape: GemmaShape = GEMMA_300M, device="cuda",
                 prefix: str = EXPERT_PREFIX):
        self.shape = shape
        self.device = torch.device(device)
        self.prefix = prefix
        self.layers: List[Dict[str, torch.Tensor]] = []
        bf = dict(dtype=torch.bfloat16, device=self.device)
        f32 = dict(dtype=torch.float32, device=self.device)
        for i in range(shape.depth):
            p = f"{prefix}layers.{i}."
            self.layers.append({
                "w_qkv": torch.empty((shape.qkv_dim, shape.width), **bf),
                "w_o": torch.empty((shape.width, shape.q_dim), **bf),
                "w_gate": torch.empty((shape.mlp_dim, shape.width), **bf),
                "w_up": torch.empty((shape.mlp_dim, shape.width), **bf),
                "w_down": torch.empty((shape.width, shape.mlp_dim), **bf),
            })
        n_norm = 2 * shape.depth + 1
        self.n_norm = n_norm
        self.w_dense = torch.empty((n_norm * 3 * shape.width, shape.width), **f32)
        self.b_dense = torch.empty((n_norm * 3 * shape.width,), **f32)
        self.glue = {k: None for k in ("action_in_proj.weight", "action_in_proj.bias", "action_out_proj.weight",
                                       "action_out_proj.bias", "time_mlp_in.weight", "time_mlp_in.bias",
                                       "time_mlp_out.weight", "time_mlp_out.bias")}
        self.load(sd)

    def load(self, sd: Dict[str, torch.Tensor]) -> None:
        """(Re)pack from a state dict IN PLACE: device addresses never change, so a
        captured graph stays valid (``modeling_gemma.py:627-652``)."""
        s = self.shape
        for i, L in enumerate(self.layers):
            p = f"{self.prefix}layers.{i}."
            L["w_qkv"].copy_(torch.cat([sd[p + "self_attn.q_proj.weight"], sd[p + "self_attn.k_proj.weight"],
                                        sd[p + "self_attn.v_proj.weight"]], 0))
            L["w_o"].copy_(sd[p + "self_attn.o_proj.weight"])
            L["w_gate"].copy_(sd[p + "mlp.gate_proj.weight"])
            L["w_up"].copy_(sd[p + "mlp.up_proj.weight"])
            L["w_down"].copy_(sd[p + "mlp.down_proj.weight"])
        keys = []
        for i in range(s.depth):
            keys += [f"{self.prefix}layers.{i}.input_layernorm.dense", f"{self.prefix}layers.{i}.post_attention_layernorm.dense"]
        keys.append(f"{self.prefix}norm.dense")
        rows = 3 * s.width
        for j, k in enumerate(keys):
            self.w_dense[j * rows:(j + 1) * rows].copy_(sd[k + ".weight"])
            self.b_dense[j * rows:(j + 1) * rows].copy_(sd[k + ".bias"])
        for k in self.glue:
            t = sd[k].to(device=self.device, dtype=torch.float32).contiguous()
            if self.glue[k] is None:
                self.glue[k] = t
            else:
                self.glue[k].copy_(t)

    def nbytes_streamed_per_step(self) -> int:
        """Weight bytes one denoise step reads (GEMM weights only)."""
        return sum(t.numel() * t.element_size() for L in self.layers for t in L.values())


class DenoiseRunner:
    """Static buffers + C plan for the ``num_steps`` Euler loop of ``batch`` observations.

    With ``batch`` B > 1 the observations are denoised together: every GEMM runs
    over B x horizon token rows (the weights stream once per step for all of them),
    attention runs per observation over its own KV cache, and the per-layer caches
    hold B caches back to back (``cache(i, b)`` is observation b's view)."""

    def __init__(self, weights: ExpertWeights, prefix_len: int, num_steps: int = 10, horizon: int = 50,
                 action_dim: int = 32, attn_splits: int = 0, batch: int = 1,
                 fold_source: Optional["DenoiseRunner"] = None, noise_method: str = "flow_ode",
                 noise_level: float = 0.0):
        self.w = weights
        s = weights.shape
        dev = weights.device
        self.device = dev
        self.prefix_len = prefix_len
        self.num_steps = num_steps
        self.horizon = horizon
        self.action_dim = action_dim
        self.batch = batch
        self.kv_rows = prefix_len + horizon
        m = horizon * batch  # token rows of every GEMM
        self.rows = m
        bf = dict(dtype=torch.bfloat16, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        # [batch * hkv, kv_rows, d] per layer (hkv = 1): observation b's cache is row block b
        self.k_cache = [torch.zeros((batch * s.num_kv_heads, self.kv_rows, s.head_dim), **bf) for _ in range(s.depth)]
        self.v_cache = [torch.zeros((batch * s.num_kv_heads, self.kv_rows, s.head_dim), **bf) for _ in range(s.depth)]
        self.key_valid = torch.ones(batch * self.kv_rows, dtype=torch.uint8, device=dev)
        self.inv_freq = rope_inv_freq(s.head_dim, s.rope_base, dev)
        self.rope_cos = torch.empty((m, s.head_dim), **bf)
        self.rope_sin = torch.empty((m, s.head_dim), **bf)
        self.h = torch.zeros((m, s.width), **bf)
        self.xn = torch.zeros((m, s.width), **bf)
        self.q = torch.zeros((m, s.num_heads, s.head_dim), **bf)
        self.attn = torch.zeros((m, s.q_dim), **bf)
        self.act = torch.zeros((m, s.mlp_dim), **bf)
        self.x_t = torch.zeros((m, action_dim), **f32)
        self.v_t = torch.zeros((m, action_dim), **f32)
        self.kv_stage = torch.zeros((2, m, s.head_dim), **bf) if batch > 1 else None
        # Sampler: flow_ode (the reference engine's) or a stochastic one, whose per-step
        # N(0, 1) noise lives in step_noise (redrawn by draw_step_noise before a call).
        self.noise_method = noise_method
        self.coefs = sampler_coefs(num_steps, noise_method, noise_level)
        self.stochastic = noise_method != "flow_ode"
        self.step_noise = torch.zeros((num_steps, m, action_dim), **f32) if self.stochastic else None
        self.ws = ops.workspace(dev)
        self.ts = timesteps(num_steps)
        self._host_ts = (ctypes.c_float * (num_steps + 1))(*[float(v) for v in self.ts])
        self.table = torch.empty((num_steps, weights.n_norm * 3 * s.width), **f32)
        # Folded norms (default for <= 64 tokens per observation, PI05_FOLD_NORM=0 to keep the norm
        # kernels): per step and layer, q|k|v and gate/up with that step's
        # input_layernorm / post_attention_layernorm (1 + scale) folded into their
        # columns, plus the biases W . shift (pi05_fold_adarms).  The step's
        # weight stream keeps its size; the copies cost num_steps x 22 MB per layer
        # of HBM (4 GB for the 10-step Gemma-300M loop).
        self.fold = None
        self._fold_owner = fold_source is None
        if fold_source is not None:
            # the folded copies depend on the weights and timesteps only: share them
            self.fold = fold_source.fold
        elif horizon <= 64 and os.environ.get("PI05_FOLD_NORM", "1") != "0":
            n = num_steps * s.depth
            self.fold = {
                "w_qkv": torch.empty((n, s.qkv_dim, s.width), **bf),
                "w_gate": torch.empty((n, s.mlp_dim, s.width), **bf),
                "w_up": torch.empty((n, s.mlp_dim, s.width), **bf),
                "b_qkv": torch.empty((n, s.qkv_dim), **f32),
                "b_gate": torch.empty((n, s.mlp_dim), **f32),
                "b_up": torch.empty((n, s.mlp_dim), **f32),
            }
        self.build_table()
        self._layers = (abi.Pi05ExpertLayer * s.depth)()
        for i, L in enumerate(weights.layers):
            self._layers[i] = abi.Pi05ExpertLayer(L["w_qkv"].data_ptr(), L["w_o"].data_ptr(), L["w_gate"].data_ptr(),
                                                  L["w_up"].data_ptr(), L["w_down"].data_ptr(),
                                                  self.k_cache[i].data_ptr(), self.v_cache[i].data_ptr())
        g = weights.glue
        self.plan = abi.Pi05ExpertPlan(
            depth=s.depth, width=s.width, mlp_dim=s.mlp_dim, n_q_heads=s.num_heads, n_kv_heads=s.num_kv_heads,
            head_dim=s.head_dim, tokens=horizon, action_dim=action_dim, prefix_len=prefix_len, kv_rows=self.kv_rows,
            eps=s.rms_eps, layers=ctypes.cast(self._layers, ctypes.POINTER(abi.Pi05ExpertLayer)),
            num_steps=num_steps, host_timesteps=ctypes.cast(self._host_ts, ctypes.POINTER(ctypes.c_float)),
            mod_table=self.table.data_ptr(), w_in=g["action_in_proj.weight"].data_ptr(),
            b_in=g["action_in_proj.bias"].data_ptr(), w_out=g["action_out_proj.weight"].data_ptr(),
            b_out=g["action_out_proj.bias"].data_ptr(), rope_cos=self.rope_cos.data_ptr(),
            rope_sin=self.rope_sin.data_ptr(), key_valid=self.key_valid.data_ptr(), x_t=self.x_t.data_ptr(),
            v_t=self.v_t.data_ptr(), h=self.h.data_ptr(), xn=self.xn.data_ptr(), q=self.q.data_ptr(),
            attn=self.attn.data_ptr(), act=self.act.data_ptr(), workspace=self.ws.data_ptr(),
            workspace_bytes=self.ws.numel(), attn_splits=attn_splits, batch=batch,
            kv_stage=self.kv_stage.data_ptr() if self.kv_stage is not None else None,
            step_noise=self.step_noise.data_ptr() if self.step_noise is not None else None)
        if self.stochastic:
            self._host_coefs = (ctypes.c_float * self.coefs.numel())(*[float(v) for v in self.coefs.flatten()])
            self.plan.host_step_coefs = ctypes.cast(self._host_coefs, ctypes.POINTER(ctypes.c_float))
        if self.fold is not None:
            fd = self.fold
            self._fold = (abi.Pi05ExpertFold * (num_steps * s.depth))()
            for i in range(num_steps * s.depth):
                self._fold[i] = abi.Pi05ExpertFold(*(fd[k][i].data_ptr() for k in
                                                     ("w_qkv", "w_gate", "w_up", "b_qkv", "b_gate", "b_up")))
            self.plan.fold = ctypes.cast(self._fold, ctypes.POINTER(abi.Pi05ExpertFold))
        self.graph: Optional[torch.cuda.CUDAGraph] = None

    def build_table(self) -> None:
        """The adaRMS modulation table for every step, on device (engine.py:556-599)."""
        s = self.w.shape
        g = self.w.glue
        ts_dev = self.ts[: self.num_steps].to(self.device)
        abi.adarms_table(ts_dev, s.width, g["time_mlp_in.weight"], g["time_mlp_in.bias"], g["time_mlp_out.weight"],
                         g["time_mlp_out.bias"], self.w.w_dense, self.w.b_dense, self.w.n_norm, self.table, self.ws)
        self.build_fold()

    def build_fold(self) -> None:
        """Fold every step's layer norms into the q|k|v and gate/up copies, in place
        (after the table; a captured graph keeps its addresses).  A runner that shares
        another's copies leaves them to their owner."""
        if self.fold is None or not self._fold_owner:
            return
        s = self.w.shape
        W = s.width
        tab = self.table.view(self.num_steps, self.w.n_norm, 3, W)  # [scale | shift | gate] per norm
        fd = self.fold
        for st in range(self.num_steps):
            for l, L in enumerate(self.w.layers):
                i = st * s.depth + l
                m1, m2 = tab[st, 2 * l], tab[st, 2 * l + 1]  # input_layernorm, post_attention_layernorm
                abi.fold_adarms(L["w_qkv"], m1[0], m1[1], fd["w_qkv"][i], fd["b_qkv"][i])
                abi.fold_adarms(L["w_gate"], m2[0], m2[1], fd["w_gate"][i], fd["b_gate"][i])
                abi.fold_adarms(L["w_up"], m2[0], m2[1], fd["w_up"][i], fd["b_up"][i])

    def cache(self, i: int, b: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
        """Layer i's (K, V) cache of observation b, ``[1, kv_rows, d]`` views."""
        return self.k_cache[i][b: b + 1], self.v_cache[i][b: b + 1]

    def key_valid_of(self, b: int = 0) -> torch.Tensor:
        return self.key_valid[b * self.kv_rows: (b + 1) * self.kv_rows]

    def set_prefix(self, kv: Sequence[Tuple[torch.Tensor, torch.Tensor]], prefix_valid: torch.Tensor,
                   b: int = 0) -> None:
        """Fill the prefix rows of every layer's static KV buffer (``prime_kv_static``)
        and the key mask of observation b; ``kv[i]`` = (K, V) ``[P, 256]`` (any
        leading 1-dims)."""
        p = self.prefix_len
        for i, (k, v) in enumerate(kv):
            kc, vc = self.cache(i, b)
            kc[0, :p].copy_(k.reshape(p, -1))
            vc[0, :p].copy_(v.reshape(p, -1))
        kvld = self.key_valid_of(b)
        kvld[:p].copy_(prefix_valid.reshape(-1).to(torch.uint8))
        kvld[p:].fill_(1)

    def _enqueue(self, stream: int) -> None:
        s = self.w.shape
        hz = self.horizon
        for b in range(self.batch):
            abi.rope_table(self.key_valid_of(b), self.prefix_len, 1, hz, self.inv_freq, s.head_dim,
                           self.rope_cos[b * hz: (b + 1) * hz], self.rope_sin[b * hz: (b + 1) * hz], stream)
        abi.denoise_loop(self.plan, stream)

    def draw_step_noise(self, generator: Optional[torch.Generator] = None) -> None:
        """Fresh N(0, 1) noise for every step of a stochastic sampler (the reference
        draws ``sample_noise(x_t.shape)`` once per step, ``engine.py:395-402``)."""
        if self.step_noise is not None:
            self.step_noise.normal_(generator=generator)

    def run(self, noise: torch.Tensor, use_graph: bool = True,
            step_noise: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Run the loop from ``noise`` [batch * 50, 32] (any leading shape); returns the
        actions (a view of the static buffer, [batch * 50, 32]).  A stochastic sampler
        uses ``step_noise`` [num_steps, batch * 50, 32] when given, else fresh noise."""
        self.x_t.copy_(noise.reshape(self.rows, self.action_dim))
        if self.step_noise is not None:
            if step_noise is not None:
                self.step_noise.copy_(step_noise.reshape(self.step_noise.shape))
            else:
                self.draw_step_noise()
        if use_graph:
            if self.graph is None:
                self.capture()
            self.graph.replay()
        else:
            self._enqueue(abi.stream_of(self.device))
        return self.x_t

    def capture(self) -> None:
        # Warm up (function attributes, lazy module loading) outside the capture.
        saved = self.x_t.clone()
        self._enqueue(abi.stream_of(self.device))
        torch.cuda.synchronize(self.device)
        self.x_t.copy_(saved)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._enqueue(torch.cuda.current_stream(self.device).cuda_stream)
        self.graph = g
