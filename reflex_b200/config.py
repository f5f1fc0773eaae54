"""Dimensions and switches of the action expert served by the engine.

Defaults follow PI05ActionExpertConfig (reflex/policies/pi05/configuration_pi05.py:79-91:
Gemma-300M, width 1024, 8 x 256 heads, 1 KV head, GeGLU MLP 4096, 18 layers)
and PI05Config (:107-126: chunk 50, action/state dim 32, 10 steps, periods
4e-3..4).  ``adarms`` selects the norm:

* ``"gate"`` — the in-tree AdaRMSNorm (reflex/policies/pi05/modeling_pi05.py:50-99):
  y = w * rmsnorm(x) * m, residual gate = m, m = dense(cond) of width W.
* ``"ssg"``  — scale/shift/gate adaRMS: y = rmsnorm(x) * (1 + scale) + shift,
  residual gate = gate, [scale|shift|gate] = dense(cond) of width 3W.
* ``"none"`` — PI0 (reflex/policies/pi0): AdaRMSNorm without conditioning,
  y = w * rmsnorm(x), residual gate 1.
"""
from __future__ import annotations

from dataclasses import dataclass, replace


@dataclass(frozen=True)
class ExpertConfig:
    variant: str = "pi05"  # "pi05" or "pi0"
    num_layers: int = 18
    width: int = 1024
    num_heads: int = 8
    num_kv_heads: int = 1
    head_dim: int = 256
    mlp_dim: int = 4096
    action_dim: int = 32
    state_dim: int = 32
    chunk_size: int = 50
    num_steps: int = 10
    min_period: float = 4e-3
    max_period: float = 4.0
    rope_theta: float = 10000.0
    max_position_embeddings: int = 8192
    eps: float = 1e-6
    adarms: str = "ssg"  # "gate" | "ssg" | "none"
    quant_mode: str = "i8_sym"  # "i8_sym" | "u8_ref"

    @property
    def suffix_len(self) -> int:
        """Suffix tokens per stream: PI0 prepends one state token."""
        return self.chunk_size + (1 if self.variant == "pi0" else 0)

    @property
    def n_norms(self) -> int:
        return 2 * self.num_layers + 1

    @property
    def mod_width(self) -> int:
        return 3 * self.width if self.adarms == "ssg" else self.width

    def with_(self, **kw) -> "ExpertConfig":
        return replace(self, **kw)


def pi05_config(**kw) -> ExpertConfig:
    return ExpertConfig(variant="pi05", **kw)


def pi0_config(**kw) -> ExpertConfig:
    kw.setdefault("adarms", "none")
    return ExpertConfig(variant="pi0", **kw)


def vlm_config(**kw) -> ExpertConfig:
    """The prefix (VLM) layers: Gemma-2B shapes (width 2048, 8 x 256 heads, one
    KV head, GeGLU 16384, 18 layers), RMSNorm without conditioning; the
    streaming frame update runs them over each new frame."""
    kw.setdefault("width", 2048)
    kw.setdefault("mlp_dim", 16384)
    kw.setdefault("adarms", "none")
    return ExpertConfig(variant="vlm", **kw)


def timestep_schedule(num_steps: int) -> list[float]:
    """t_0 = 1.0, t_{k+1} = fp32(t_k + fp32(-1/num_steps)) as in
    reflex/policies/pi05/modeling_pi05.py:1403-1418 (fp32 tensors)."""
    import numpy as np

    dt = np.float32(-1.0 / num_steps)
    t = np.float32(1.0)
    out = []
    for _ in range(num_steps):
        out.append(float(t))
        t = np.float32(t + dt)
    return out


@dataclass(frozen=True)
class VisionConfig:
    """The SigLIP vision tower and PaliGemma projector that turn a camera image
    into the 256 image tokens of the prefix (the ``get_image_features`` call at
    reflex/policies/pi05/modeling_pi05.py:141-158,244; PaliGemma-3B-224's
    SigLIP-So400m/14: 27 layers, width 1152, 16 x 72 heads, MLP 4304 with
    GELU-tanh, LayerNorm eps 1e-6, 14 x 14 patches of a 224 x 224 image, and a
    1152 -> 2048 projector)."""

    num_layers: int = 27
    width: int = 1152
    num_heads: int = 16
    head_dim: int = 72
    mlp_dim: int = 4304
    patch: int = 14
    image: int = 224
    channels: int = 3
    proj_dim: int = 2048
    eps: float = 1e-6

    @property
    def grid(self) -> int:
        return self.image // self.patch

    @property
    def tokens(self) -> int:
        """Image tokens (patches) per image."""
        return self.grid * self.grid

    @property
    def patch_dim(self) -> int:
        return self.channels * self.patch * self.patch

    def with_(self, **kw) -> "VisionConfig":
        return replace(self, **kw)
