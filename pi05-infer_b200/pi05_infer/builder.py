"""``build_model`` / ``get_model`` with the reference's signatures (``builder.py:34-151``).

Loads a pi0.5 checkpoint (``*.safetensors`` or an FSDP ``full_weights.pt``, as the
reference's builder does, ``builder.py:77-106``) into an ``OpenPi0Inference``.
openpi's data configs and input/output transforms are out of scope, so
``config_name`` only selects the model family (pi0.5 variants) and
``data_kwargs`` is accepted and ignored.
"""

from __future__ import annotations

import glob
import os
from typing import Any, Dict, Optional

import torch

from .config import EngineConfig
from .engine import OpenPi0Inference

SUPPORTED_CONFIGS = ("pi05_libero", "pi05_turtle", "pi05")


def _load_state_dict(model_path: str) -> Dict[str, torch.Tensor]:
    if os.path.isdir(model_path):
        files = sorted(glob.glob(os.path.join(model_path, "*.safetensors")))
        if files:
            from safetensors.torch import load_file

            sd: Dict[str, torch.Tensor] = {}
            for f in files:
                sd.update(load_file(f))
            return sd
        pt = os.path.join(model_path, "full_weights.pt")
        if os.path.exists(pt):
            model_path = pt
        else:
            raise FileNotFoundError(f"no *.safetensors or full_weights.pt under {model_path}")
    obj = torch.load(model_path, map_location="cpu", weights_only=True)
    if isinstance(obj, dict) and "state_dict" in obj and isinstance(obj["state_dict"], dict):
        obj = obj["state_dict"]
    # FSDP / wrapper prefixes (builder.py:88-101)
    out = {}
    for k, v in obj.items():
        for pre in ("module.", "model.", "_orig_mod."):
            if k.startswith(pre) and not k.startswith("model.layers"):
                k = k[len(pre):]
        out[k] = v
    return out


def build_model(model_path: str, config_name: str = "pi05_libero", *, data_kwargs: Optional[dict] = None,
                **overrides: Any) -> OpenPi0Inference:
    """Build the inference engine from a checkpoint (``builder.py:34-138``)."""
    del data_kwargs
    if config_name not in SUPPORTED_CONFIGS:
        raise ValueError(f"config {config_name!r} not supported (pi0.5 variants only: {SUPPORTED_CONFIGS})")
    cfg = EngineConfig()
    device = overrides.pop("device", "cuda")
    for k, v in overrides.items():
        if not hasattr(cfg, k):
            raise TypeError(f"unknown override {k!r}")
        setattr(cfg, k, v)
    sd = _load_state_dict(model_path)
    return OpenPi0Inference(cfg, sd, device=device)


def get_model(cfg: Any, torch_dtype=None) -> OpenPi0Inference:  # noqa: ARG001
    """``get_model(cfg)`` (``builder.py:141-151``): ``cfg`` carries ``model_path`` / ``config_name``."""
    get = cfg.get if isinstance(cfg, dict) else (lambda k, d=None: getattr(cfg, k, d))
    return build_model(get("model_path"), get("config_name", "pi05_libero"))
