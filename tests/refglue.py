"""Adapters over ``baseline/ref_pipeline.py`` (the reference's own ``GemmaModel``
loaded from ``baseline/_ref``, plus the restated glue) for the tests that run the
reference's action expert.  Test infrastructure only."""

from __future__ import annotations

import importlib.util
import os
import sys

import torch

from pi05_infer import synthetic

_REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _pipeline():
    name = "pi05_ref_pipeline"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(name, os.path.join(_REPO, "baseline", "ref_pipeline.py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return sys.modules[name]


def build_expert(mod, ref_loader, w, shape, depth, dtype, device="cpu"):  # noqa: ARG001
    """The reference expert ``GemmaModel`` (``mod``) with weights ``w``."""
    return _pipeline().build_gemma(mod, dict(w), synthetic.EXPERT_PREFIX, shape, depth, True, dtype, device)


def velocity(model, w, x_t, t, kv, prefix_pad, dtype, device="cpu", static_kv=False):
    """v_t ``[1, M, 32]`` through the reference model (see ``ref_pipeline.velocity``)."""
    pkv = [(k.to(device, dtype), v.to(device, dtype)) for k, v in kv]
    return _pipeline().velocity(model, w, x_t, t, pkv, prefix_pad, device=device, static_kv=static_kv)
