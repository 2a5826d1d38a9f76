"""Static shapes of pi0.5 and the engine config.

The two Gemma variants follow openpi's ``gemma_2b`` (PaliGemma prefix LM) and
``gemma_300m`` (action expert) as instantiated by
``pi05_infer/openpi_patched/gemma_pytorch.py:33-82`` of the reference; the SigLIP
So400m/14 tower follows the HF PaliGemma vision config set there (intermediate
4304, projection 2048).  ``EngineConfig`` mirrors ``OpenPi0InferConfig``
(``pi05_infer/engine.py:120-140``): ``num_steps``, ``action_horizon``,
``action_dim``, ``action_chunk``.
"""

from __future__ import annotations

import dataclasses


@dataclasses.dataclass(frozen=True)
class GemmaShape:
    width: int
    depth: int
    mlp_dim: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    rms_eps: float = 1e-6
    rope_base: float = 10000.0

    @property
    def q_dim(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return (self.num_heads + 2 * self.num_kv_heads) * self.head_dim


@dataclasses.dataclass(frozen=True)
class SiglipShape:
    width: int = 1152
    depth: int = 27
    mlp_dim: int = 4304
    num_heads: int = 16
    head_dim: int = 72
    patch: int = 14
    image_size: int = 224
    proj_dim: int = 2048
    ln_eps: float = 1e-6

    @property
    def num_patches(self) -> int:
        return (self.image_size // self.patch) ** 2


GEMMA_300M = GemmaShape(width=1024, depth=18, mlp_dim=4096, num_heads=8, num_kv_heads=1, head_dim=256)
GEMMA_2B = GemmaShape(width=2048, depth=18, mlp_dim=16384, num_heads=8, num_kv_heads=1, head_dim=256)
SIGLIP_SO400M = SiglipShape()

VOCAB_SIZE = 257152
ACTION_DIM = 32
ACTION_HORIZON = 50
# adaRMS: two norms per expert layer plus the final norm.
def num_adarms_norms(expert: GemmaShape) -> int:
    return 2 * expert.depth + 1


@dataclasses.dataclass
class EngineConfig:
    """Mirror of ``OpenPi0InferConfig`` (reference ``pi05_infer/engine.py:120-140``)."""

    num_steps: int = 10
    action_horizon: int = ACTION_HORIZON
    action_dim: int = ACTION_DIM
    action_chunk: int = ACTION_HORIZON
    # Sampler of the Euler loop: "flow_ode" (deterministic, the reference engine's) or
    # the stochastic "flow_sde" / "flow_cps" with this noise level.
    noise_level: float = 0.0
    noise_method: str = "flow_ode"
    expert: GemmaShape = GEMMA_300M
    prefix_lm: GemmaShape = GEMMA_2B
    siglip: SiglipShape = SIGLIP_SO400M
    max_prefix_len: int = 1480
    # Input / output transforms of predict_action_batch (openpi data config):
    # "libero" (main + wrist camera, 7 action dims), "turtle" (main + up to two
    # extra views, 6 action dims) or "none" (32 action dims, no camera mapping);
    # quantile normalisation as openpi uses it for pi0.5.
    policy: str = "libero"
    use_quantile_norm: bool = True

    @property
    def env_action_dim(self) -> int:
        return {"libero": 7, "turtle": 6}.get(self.policy, self.action_dim)
