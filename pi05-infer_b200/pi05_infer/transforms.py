"""Observation preprocessing and the action output transform, on the GPU.

``predict_action_batch`` of the reference (``engine.py:321-342``) wraps
``sample_actions`` in openpi's input transforms (image parsing and resizing,
``Normalize`` of the state, padding to the model's action dimension) and output
transforms (``Unnormalize`` of the actions, the policy's slice to the robot's
action dimension, e.g. ``LiberoOutputs`` ``[:, :7]``), built from the checkpoint's
norm statistics (``builder.py:120-136``).  Those run per sample on the host in
numpy there; here they are three small kernels of the C ABI
(``pi05_preprocess_images``, ``pi05_normalize_rows``, ``pi05_unnormalize_rows``).

Prompt tokenisation (sentencepiece) stays with the caller: the observation
carries ``tokenized_prompt`` / ``tokenized_prompt_mask``.
"""

from __future__ import annotations

import dataclasses
import json
import os
from typing import Dict, Optional

import torch

from . import _lib, abi


@dataclasses.dataclass
class NormStats:
    """Per-feature statistics of one array (openpi ``NormStats``): mean/std, and
    the 1 % / 99 % quantiles used when ``use_quantiles``."""

    mean: torch.Tensor
    std: torch.Tensor
    q01: Optional[torch.Tensor] = None
    q99: Optional[torch.Tensor] = None

    @classmethod
    def from_dict(cls, d: Dict) -> "NormStats":
        def t(k):
            return None if d.get(k) is None else torch.tensor(d[k], dtype=torch.float32)

        return cls(t("mean"), t("std"), t("q01"), t("q99"))

    def pair(self, use_quantiles: bool):
        """(a, b, mode) for the kernels: (mean, std, 0) or (q01, q99, 1)."""
        if use_quantiles:
            if self.q01 is None or self.q99 is None:
                raise ValueError("quantile normalisation needs q01 / q99 statistics")
            return self.q01, self.q99, 1
        return self.mean, self.std, 0


def load_norm_stats(path: str) -> Dict[str, NormStats]:
    """``norm_stats.json`` as openpi writes it: ``{"norm_stats": {key: {mean, std,
    q01, q99}}}``; ``path`` is the file or a directory searched for it."""
    if os.path.isdir(path):
        found = None
        for root, _, files in os.walk(path):
            if "norm_stats.json" in files:
                found = os.path.join(root, "norm_stats.json")
                break
        if found is None:
            raise FileNotFoundError(f"no norm_stats.json under {path}")
        path = found
    with open(path) as f:
        d = json.load(f)
    d = d.get("norm_stats", d)
    return {k: NormStats.from_dict(v) for k, v in d.items()}


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def preprocess_images(images: torch.Tensor, size: int = 224, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """uint8 ``[n, h, w, 3]`` (or ``[n, 3, h, w]``) on the GPU -> fp32 ``[n, 3, size, size]``
    in [-1, 1], resized with padding (aspect ratio kept, border -1)."""
    if images.dtype != torch.uint8 or not images.is_cuda or images.dim() != 4:
        raise ValueError("expected a uint8 CUDA tensor [n, h, w, 3] or [n, 3, h, w]")
    images = images.contiguous()
    chw = images.shape[1] == 3 and images.shape[-1] != 3
    n = images.shape[0]
    h, w = (images.shape[2], images.shape[3]) if chw else (images.shape[1], images.shape[2])
    if out is None:
        out = torch.empty((n, 3, size, size), dtype=torch.float32, device=images.device)
    abi._bind()
    _lib.call("pi05_preprocess_images", images.data_ptr(), n, h, w, 1 if chw else 0, out.data_ptr(), size,
              _stream(images.device))
    return out


def normalize_state(state: torch.Tensor, stats: Optional[NormStats], use_quantiles: bool, dim: int) -> torch.Tensor:
    """``[B, s]`` fp32 state -> ``[B, dim]`` normalised and zero-padded."""
    x = state.to(torch.float32).contiguous()
    rows, din = x.shape
    out = torch.empty((rows, dim), dtype=torch.float32, device=x.device)
    a = b = None
    nstat, mode = 0, 0
    if stats is not None:
        a, b, mode = stats.pair(use_quantiles)
        nstat = min(a.numel(), din)
        a = a.to(x.device).contiguous()
        b = b.to(x.device).contiguous()
    abi._bind()
    _lib.call("pi05_normalize_rows", x.data_ptr(), rows, din, abi.ptr(a), abi.ptr(b), nstat, mode, out.data_ptr(),
              dim, _stream(x.device))
    return out


def unnormalize_actions(actions: torch.Tensor, stats: Optional[NormStats], use_quantiles: bool,
                        out_dim: int) -> torch.Tensor:
    """``[B, T, D]`` fp32 actions -> ``[B, T, out_dim]`` un-normalised (the first
    ``out_dim`` features)."""
    x = actions.to(torch.float32).contiguous()
    din = x.shape[-1]
    rows = x.numel() // din
    out = torch.empty((*x.shape[:-1], out_dim), dtype=torch.float32, device=x.device)
    a = b = None
    nstat, mode = 0, 0
    if stats is not None:
        a, b, mode = stats.pair(use_quantiles)
        nstat = min(a.numel(), din)
        a = a.to(x.device).contiguous()
        b = b.to(x.device).contiguous()
    abi._bind()
    _lib.call("pi05_unnormalize_rows", x.data_ptr(), rows, din, abi.ptr(a), abi.ptr(b), nstat, mode,
              out.data_ptr(), out_dim, _stream(x.device))
    return out
