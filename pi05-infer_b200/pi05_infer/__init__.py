"""pi05_infer on B200: pi0.5 ``sample_actions`` with hand-written sm_100a kernels.

Drop-in for the reference package's engine/builder API (``build_model``,
``get_model``, ``Engine``/``OpenPi0Inference``, ``EngineConfig``) and its custom
ops ``torch.ops.pi05_infer.gate_up_geglu`` / ``qkv_rope_kv``.
"""

from .config import EngineConfig
from .engine import Engine, Observation, OpenPi0Inference
from .builder import build_model, get_model
from . import ops  # registers torch.ops.pi05_infer.*

__all__ = ["build_model", "get_model", "Engine", "EngineConfig", "OpenPi0Inference", "Observation", "ops"]
