"""Load modules of the unmodified reference package installed under ``baseline/_ref``.

``baseline/_ref`` holds the reference (``chenchaoxu7575/pi05-infer``) installed with
``pip install --no-index --no-build-isolation --no-deps --ignore-requires-python
--target baseline/_ref <copy of the reference>``.  Its package cannot be imported
as a whole here (``pi05_infer/__init__.py`` imports openpi, which is absent), so
this module loads single files of it under a private package name:

* ``load_modeling_gemma(fused_ops=...)``: the vendored action-expert / Gemma
  module ``pi05_infer/gemma/modeling_gemma.py`` with the two shims it needs under
  transformers 5.x (a ``LossKwargs`` TypedDict and the ``"default"`` RoPE init).
  Its optional ``from . import rlinf_fused_denoise`` is resolved to ``fused_ops``
  when one is given (a module object, e.g. ``pi05_infer.ops``), to the reference's
  own Triton module when ``fused_ops="reference"``, and left unresolvable (the
  reference then runs its eager path) when ``fused_ops`` is None.
* ``load_fused_denoise()``: the reference's Triton module
  ``pi05_infer/gemma/rlinf_fused_denoise.py``.  Importing it registers
  ``torch.ops.pi05_infer.gate_up_geglu`` / ``qkv_rope_kv`` and so replaces this
  repository's registrations of the same names in that process: load it only in a
  process of its own.

Test and benchmark infrastructure only; the product never imports it.
"""

from __future__ import annotations

import importlib.util
import os
import sys
import types
import typing

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF_ROOT = os.path.join(HERE, "_ref")
_PKG = "_pi05_reference"


def available(root: str = REF_ROOT) -> bool:
    return os.path.exists(os.path.join(root, "pi05_infer", "gemma", "modeling_gemma.py"))


def _shims() -> None:
    import transformers.utils as tu
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS

    if not hasattr(tu, "LossKwargs"):
        class LossKwargs(typing.TypedDict, total=False):
            pass

        tu.LossKwargs = LossKwargs

    if "default" not in ROPE_INIT_FUNCTIONS:
        def _default_rope(config, device=None, *args, **kwargs):
            base = getattr(config, "rope_theta", None) or 10000.0
            dim = config.head_dim
            inv = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.int64).float() / dim))
            return inv, 1.0

        ROPE_INIT_FUNCTIONS["default"] = _default_rope


def _package(name: str) -> types.ModuleType:
    pkg = types.ModuleType(name)
    pkg.__path__ = []
    sys.modules[name] = pkg
    return pkg


def _exec(modname: str, path: str) -> types.ModuleType:
    spec = importlib.util.spec_from_file_location(modname, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[modname] = mod
    spec.loader.exec_module(mod)
    return mod


def load_fused_denoise(root: str = REF_ROOT) -> types.ModuleType:
    """The reference's Triton kernels and custom ops (``rlinf_fused_denoise.py``)."""
    if not available(root):
        raise FileNotFoundError(f"reference not installed under {root}")
    name = f"{_PKG}_k"
    _package(name)
    return _exec(f"{name}.rlinf_fused_denoise", os.path.join(root, "pi05_infer", "gemma", "rlinf_fused_denoise.py"))


def load_modeling_gemma(fused_ops=None, root: str = REF_ROOT, tag: str = "") -> types.ModuleType:
    """The reference's ``modeling_gemma`` module (see the module docstring for
    ``fused_ops``).  ``tag`` keeps several loads apart in one process."""
    if not available(root):
        raise FileNotFoundError(f"reference not installed under {root}")
    _shims()
    kind = "eager" if fused_ops is None else ("ref" if fused_ops == "reference" else "sub")
    name = f"{_PKG}_{kind}{tag}"
    _package(name)
    if fused_ops == "reference":
        sys.modules[f"{name}.rlinf_fused_denoise"] = load_fused_denoise(root)
    elif fused_ops is not None:
        sys.modules[f"{name}.rlinf_fused_denoise"] = fused_ops
    return _exec(f"{name}.modeling_gemma", os.path.join(root, "pi05_infer", "gemma", "modeling_gemma.py"))


def gemma_config(width: int, depth: int, mlp_dim: int, num_heads: int = 8, num_kv_heads: int = 1,
                 head_dim: int = 256, adarms: bool = True):
    """The transformers ``GemmaConfig`` the reference builds for the action expert
    (``adarms=True``) or the PaliGemma language model (``adarms=False``)."""
    from transformers.models.gemma.configuration_gemma import GemmaConfig

    cfg = GemmaConfig(head_dim=head_dim, hidden_size=width, intermediate_size=mlp_dim, num_attention_heads=num_heads,
                      num_hidden_layers=depth, num_key_value_heads=num_kv_heads, vocab_size=8,
                      hidden_activation="gelu_pytorch_tanh", use_adarms=adarms,
                      adarms_cond_dim=width if adarms else None)
    cfg._attn_implementation = "eager"
    return cfg
