"""``build_model`` / ``get_model`` with the reference's signatures (``builder.py:34-151``).

Loads a pi0.5 checkpoint (``*.safetensors`` or an FSDP ``full_weights.pt``, as the
reference's builder does, ``builder.py:77-106``) into an ``OpenPi0Inference``,
with the checkpoint's ``norm_stats.json`` (``builder.py:112-136``) when present.
``config_name`` selects the policy's input/output transform (``pi05_libero``: main
+ wrist camera, 7 action dims; ``pi05_turtle``: main + extra views, 6 action dims;
``pi05``: none); openpi's other data-config options are out of scope, so
``data_kwargs`` is accepted and ignored.
"""

from __future__ import annotations

import glob
import os
from typing import Any, Dict, Optional

import torch

from .config import EngineConfig
from .engine import OpenPi0Inference
from .transforms import load_norm_stats

SUPPORTED_CONFIGS = ("pi05_libero", "pi05_turtle", "pi05")
_POLICY = {"pi05_libero": "libero", "pi05_turtle": "turtle", "pi05": "none"}


def _load_state_dict(model_path: str) -> Dict[str, torch.Tensor]:
    """The checkpoint's state dict, searched in the reference's order
    (``builder.py:77-106``): an FSDP ``model_state_dict/full_weights.pt``, then
    ``actor/model_state_dict/full_weights.pt``, then ``*.safetensors`` files; a path
    to a single ``.pt`` / ``.safetensors`` file is also accepted."""
    path = model_path
    if os.path.isdir(model_path):
        for cand in (os.path.join(model_path, "model_state_dict", "full_weights.pt"),
                     os.path.join(model_path, "actor", "model_state_dict", "full_weights.pt"),
                     os.path.join(model_path, "full_weights.pt")):
            if os.path.exists(cand):
                path = cand
                break
        else:
            files = sorted(glob.glob(os.path.join(model_path, "*.safetensors")))
            if not files:
                raise FileNotFoundError(f"no full_weights.pt or *.safetensors under {model_path}")
            from safetensors.torch import load_file

            sd: Dict[str, torch.Tensor] = {}
            for f in files:
                sd.update(load_file(f))
            return sd
    if path.endswith(".safetensors"):
        from safetensors.torch import load_file

        return load_file(path)
    obj = torch.load(path, map_location="cpu", weights_only=True)
    if isinstance(obj, dict) and "state_dict" in obj and isinstance(obj["state_dict"], dict):
        obj = obj["state_dict"]
    # FSDP / wrapper prefixes
    out = {}
    for k, v in obj.items():
        for pre in ("module.", "_orig_mod."):
            if k.startswith(pre):
                k = k[len(pre):]
        out[k] = v
    return out


def build_model(model_path: str, config_name: str = "pi05_libero", *, data_kwargs: Optional[dict] = None,
                **overrides: Any) -> OpenPi0Inference:
    """Build the inference engine from a checkpoint (``builder.py:34-138``)."""
    del data_kwargs
    if config_name not in SUPPORTED_CONFIGS:
        raise ValueError(f"config {config_name!r} not supported (pi0.5 variants only: {SUPPORTED_CONFIGS})")
    cfg = EngineConfig(policy=_POLICY[config_name])
    device = overrides.pop("device", "cuda")
    for k, v in overrides.items():
        if not hasattr(cfg, k):
            raise TypeError(f"unknown override {k!r}")
        setattr(cfg, k, v)
    sd = _load_state_dict(model_path)
    engine = OpenPi0Inference(cfg, sd, device=device)
    # norm statistics of the checkpoint (<asset_id>/norm_stats.json), when present
    if os.path.isdir(model_path):
        try:
            engine.set_norm_stats(load_norm_stats(model_path))
        except FileNotFoundError:
            pass
    return engine


def get_model(cfg: Any, torch_dtype=None) -> OpenPi0Inference:  # noqa: ARG001
    """``get_model(cfg)`` (``builder.py:141-151``): ``cfg.model_path``, ``cfg.openpi``
    (a mapping with ``config_name`` and config overrides) and ``cfg.openpi_data``;
    attribute- or dict-style ``cfg`` alike."""
    def get(k, d=None):
        return cfg.get(k, d) if isinstance(cfg, dict) else getattr(cfg, k, d)

    openpi_cfg = dict(get("openpi") or {})
    config_name = openpi_cfg.pop("config_name", None) or get("config_name", "pi05_libero")
    return build_model(get("model_path"), config_name, data_kwargs=get("openpi_data"), **openpi_cfg)
